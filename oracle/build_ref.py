"""Compile the reference's own host-runnable code into oracle/_ref/libref.so.

TEST INFRASTRUCTURE ONLY: used by tests/golden/gen_golden.py to produce golden fixtures
from the reference itself; nothing on the product path, in the GPU tests, in smoke() or in
bench.py loads it.

The reference (thrasos-g/RDNA4-GEMM-WMMA) cannot be built here as a program: it needs
hipcc/ROCm, rocBLAS and clang's ext_vector_type, and its main() uses <<<>>> launches.  Its
semantic pieces are plain C++ though, and are compiled here straight from the files under
the reference checkout, by line range (checked against the expected first line), with a
small prelude that gives the HIP built-ins a CPU meaning:
  * GEMM_Naive            mmm.cpp:52-62        the semantic definition of the GEMM
  * validateResults       mmm.cpp:1387-1407    the GEMM check (relative 1e-4)
  * validateResults       mmmTensor.cpp:278-306 the contraction check and its output remap
  * the G pack loop nest  mmmTensor.cpp:329-340 G[r][n][m][k] -> A[(m*rt+r)][(n*rt_l+k)]
The prelude defines __global__ away, makes blockIdx/threadIdx/blockDim/gridDim per-thread
variables and turns the compile-time DIM_I/J/K (mmm.cpp:13-15) into runtime variables; the
wrappers below run GEMM_Naive over its documented launch grid (16x16 blocks,
README.md:103).  The translation unit is fed to g++ on stdin: no reference source is
written anywhere; only the shared object lands in oracle/_ref/.

    python oracle/build_ref.py [--reference DIR] [--force]

The reference checkout is the directory given by --reference, else B2G_REFERENCE_DIR, else a
directory named `reference` beside this repository.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libref.so")

# (file, first line, last line, text the first line must start with)
PIECES = {
    "gemm_naive": ("mmm.cpp", 52, 62, "__global__ void GEMM_Naive("),
    "validate_gemm": ("mmm.cpp", 1387, 1407, "static bool validateResults(float *kernelC, float *rocblasC, int size)"),
    "validate_tensor": ("mmmTensor.cpp", 278, 306, "static bool validateResults(float *kernelC, float *rocblasC, int mt, int bt, int rt)"),
    "pack_g": ("mmmTensor.cpp", 329, 340, "for (int r = 0; r < rt; r++) {"),
}

PRELUDE = r"""
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
struct b2g_shim_dim3 { unsigned x, y, z; };
static thread_local b2g_shim_dim3 blockIdx, threadIdx, blockDim, gridDim;
#define __global__ static
static int DIM_I, DIM_J, DIM_K;
"""

WRAPPERS = r"""
extern "C" void ref_gemm_naive(const uint16_t* A, const uint16_t* B, float* C, int M, int N, int K) {
  DIM_I = M; DIM_J = N; DIM_K = K;
  blockDim = {16u, 16u, 1u};
  gridDim = {(unsigned)((N + 15) / 16), (unsigned)((M + 15) / 16), 1u};
  for (unsigned by = 0; by < gridDim.y; ++by)
    for (unsigned bx = 0; bx < gridDim.x; ++bx)
      for (unsigned ty = 0; ty < blockDim.y; ++ty)
        for (unsigned tx = 0; tx < blockDim.x; ++tx) {
          blockIdx = {bx, by, 0u};
          threadIdx = {tx, ty, 0u};
          GEMM_Naive(reinterpret_cast<const _Float16*>(A), reinterpret_cast<const _Float16*>(B), C);
        }
}
extern "C" int ref_validate_gemm(float* kernelC, float* refC, int size) {
  return validateResults(kernelC, refC, size) ? 1 : 0;
}
extern "C" int ref_validate_tensor(float* kernelC, float* refC, int mt, int bt, int rt) {
  return validateResults(kernelC, refC, mt, bt, rt) ? 1 : 0;
}
"""

PACK_HEAD = r"""
extern "C" void ref_pack_g(const uint16_t* G_, uint16_t* hA_, int rt_, int nt_, int mt_, int rt_l_) {
  const int rt = rt_, nt = nt_, mt = mt_, rt_l = rt_l_;
  const int DIM_K = nt * rt_l;
  const _Float16* G = reinterpret_cast<const _Float16*>(G_);
  _Float16* hA = reinterpret_cast<_Float16*>(hA_);
"""


def reference_dir(given=None):
    """The reference checkout: `given`, else B2G_REFERENCE_DIR, else `reference` beside the
    repository."""
    if given:
        return given
    env = os.environ.get("B2G_REFERENCE_DIR")
    if env:
        return env
    return os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def reference_available(ref=None):
    ref = reference_dir(ref)
    return all(os.path.exists(os.path.join(ref, f)) for f in ("mmm.cpp", "mmmTensor.cpp"))


def _piece(name, ref):
    fname, lo, hi, head = PIECES[name]
    with open(os.path.join(ref, fname)) as f:
        lines = f.read().splitlines()
    text = lines[lo - 1:hi]
    if not text or not text[0].strip().startswith(head):
        raise RuntimeError("%s:%d does not start with %r; the reference changed" % (fname, lo, head))
    # the piece must be brace-balanced
    body = "\n".join(text)
    if body.count("{") != body.count("}"):
        raise RuntimeError("%s:%d-%d is not a complete block" % (fname, lo, hi))
    return "#line %d \"%s\"\n%s\n" % (lo, fname, body)


def translation_unit(ref=None):
    ref = reference_dir(ref)
    return (PRELUDE + _piece("gemm_naive", ref) + _piece("validate_gemm", ref)
            + _piece("validate_tensor", ref) + WRAPPERS + PACK_HEAD + _piece("pack_g", ref)
            + "}\n")


def build(force=False, ref=None):
    ref = reference_dir(ref)
    if not reference_available(ref):
        raise RuntimeError("reference sources not found under %s" % ref)
    if not force and os.path.exists(LIB):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cxx = os.environ.get("CXX") or shutil.which("g++") or "c++"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-x", "c++", "-", "-o", LIB + ".tmp"]
    res = subprocess.run(cmd, input=translation_unit(ref), capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("compiling the reference pieces failed")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="the reference checkout")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ref=a.reference))
