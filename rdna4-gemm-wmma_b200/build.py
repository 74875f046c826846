"""Build libb2g_gemm.so in-tree with nvcc for sm_100a.

    python rdna4-gemm-wmma_b200/build.py [--verbose]

The library is plain nvcc output (static CUDA runtime, no framework dependency) so a C or
C++ caller can link or dlopen it directly; Python callers use b2g.py (ctypes).
"""
import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libb2g_gemm.so")
SOURCES = ["b2g_api.cu", "b2g_shard.cu"]
HEADERS = ["ptx.cuh", "gemm_sm100.cuh", "sched.h", "errors.h", "plan.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
    "-ldl",
]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "b2g_gemm.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    cmd = [nvcc()] + NVCC_FLAGS + ["-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp"]
    cmd += [os.path.join(CSRC, f) for f in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed building libb2g_gemm.so")
    os.replace(LIB + ".tmp", LIB)
    # keep the ptxas resource summary next to the build for inspection
    with open(os.path.join(HERE, "ptxas_resources.txt"), "w") as f:
        f.write("\n".join(l for l in res.stderr.splitlines() if "ptxas info" in l) + "\n")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
