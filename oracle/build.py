"""Build the CPU oracle (oracle/orc.c) into oracle/_build/liborc.so.

TEST INFRASTRUCTURE ONLY: the oracle is the checker of the CUDA library and the CPU
baseline of bench.py; the product path never loads it.

    python oracle/build.py
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liborc.so")
SRC = os.path.join(HERE, "orc.c")

# AVX2/FMA/F16C: present on every x86-64 server CPU this code is expected to meet; the
# library built here also runs on the GPU boxes' host CPUs.
CFLAGS = ["-O3", "-std=c11", "-fPIC", "-shared", "-pthread", "-mavx2", "-mfma", "-mf16c"]


def build(force=False):
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
    cmd = [cc] + CFLAGS + ["-o", LIB + ".tmp", SRC, "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("building the oracle failed")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
