"""The C++ drop-in flow on the GPU: tests/cpp/reference_flow.cpp is the reference's host flow
(host operands, cudaMalloc, cudaMemcpy, kernel launch, cudaMemcpy back) with the launch
replaced by the library's C++ wrappers, as INTEGRATION.md shows for mmm.cpp:1496 and
mmmTensor.cpp:329-369.  It is compiled here with nvcc against include/ and libb2g_gemm.so, run
as its own process, and its output is checked:

* GEMM: the golden fixtures made by the reference's own GEMM_Naive (row pitches that TMA can
  address) and seeded U[-1,1] operands at 1024^3 and 256 x 8192 x 8192 (split K) against the
  FP64 oracle, within |C - R| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|R|;
* contraction: the reference-form golden fixture (Out[m][b][r] from G[r][n][m][k] and
  Input[b][n*rt_l+k], written by the reference's own pack and validateResults) within the
  same tolerance, plus a larger seeded case against the oracle's strided contraction.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import ROOT
from gpu_util import assert_close

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="module")
def flow_exe(b2g, cuda, tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("no nvcc")
    out = tmp_path_factory.mktemp("flow") / "reference_flow"
    libdir = os.path.join(ROOT, "rdna4-gemm-wmma_b200")
    res = subprocess.run([nvcc, "-std=c++17", "-O2", os.path.join(ROOT, "tests", "cpp", "reference_flow.cpp"),
                          "-I", os.path.join(ROOT, "include"), "-L", libdir, "-lb2g_gemm",
                          "-Xlinker", "-rpath", "-Xlinker", libdir, "-o", str(out)],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return str(out)


def _run(exe, args, tmp):
    res = subprocess.run([exe] + [str(a) for a in args], capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, (res.returncode, res.stdout, res.stderr)
    assert res.stdout.startswith("ok"), res.stdout
    return res.stdout


def _gemm_via_flow(exe, tmp, A, B):
    M, K = A.shape
    N = B.shape[1]
    pa, pb, pc = tmp / "A.f16", tmp / "B.f16", tmp / "C.f32"
    np.ascontiguousarray(A).view(np.uint16).tofile(pa)
    np.ascontiguousarray(B).view(np.uint16).tofile(pb)
    _run(exe, ["gemm", M, N, K, pa, pb, pc], tmp)
    return np.fromfile(pc, dtype=np.float32).reshape(M, N)


def test_cpp_flow_gemm_golden(flow_exe, orc, tmp_path):
    z = np.load(os.path.join(GOLDEN, "gemm_naive.npz"))
    ran = 0
    for i in range(int(z["n_cases"])):
        A, B, C = z["c%d_A" % i].view(np.float16), z["c%d_B" % i].view(np.float16), z["c%d_C" % i]
        M, K = A.shape
        N = B.shape[1]
        C_got = _gemm_via_flow(flow_exe, tmp_path, A, B)
        max_a = float(np.abs(A.astype(np.float32)).max())
        max_b = float(np.abs(B.astype(np.float32)).max())
        assert_close(orc, C_got, C.astype(np.float64), K, max_a, max_b,
                     what="golden %dx%dx%d" % (M, N, K))
        ran += 1
    assert ran == int(z["n_cases"])


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (256, 8192, 8192)])
def test_cpp_flow_gemm_seeded(flow_exe, orc, tmp_path, M, N, K):
    A = orc.uniform_f16((M, K), 51)
    B = orc.uniform_f16((K, N), 52)
    C_got = _gemm_via_flow(flow_exe, tmp_path, A, B)
    rows = sorted(set([0, 1, M // 3, M // 2, M - 1]))
    for r in rows:
        assert_close(orc, C_got[r:r + 1], orc.gemm_f64(A[r:r + 1], B), K, what="row %d" % r)


def test_cpp_flow_contraction_golden_and_seeded(flow_exe, orc, tmp_path):
    z = np.load(os.path.join(GOLDEN, "contraction_ref.npz"))
    mt, rt, nt, rt_l, bt = (int(x) for x in z["dims"])
    pg, pi, po = tmp_path / "G.f16", tmp_path / "In.f16", tmp_path / "Out.f32"
    z["G"].tofile(pg)
    z["In"].tofile(pi)
    _run(flow_exe, ["contract", mt, rt, nt, rt_l, bt, pg, pi, po], tmp_path)
    out = np.fromfile(po, dtype=np.float32)
    assert_close(orc, out, z["Out"].astype(np.float64), nt * rt_l, what="golden contraction")
    # a larger reference-form case: mt=4, rt=64, nt=3, rt_l=128, bt=512
    mt, rt, nt, rt_l, bt = 4, 64, 3, 128, 512
    G = orc.uniform_f16((rt * nt * mt * rt_l,), 53)
    In = orc.uniform_f16((bt * nt * rt_l,), 54)
    G.view(np.uint16).tofile(pg)
    In.view(np.uint16).tofile(pi)
    _run(flow_exe, ["contract", mt, rt, nt, rt_l, bt, pg, pi, po], tmp_path)
    out = np.fromfile(po, dtype=np.float32)
    ref = orc.contract5d_f64(G, (mt, 1, rt, nt, rt_l), (rt_l, 0, nt * mt * rt_l, mt * rt_l, 1),
                             In, (nt, rt_l, bt), (rt_l, 1, nt * rt_l), (mt, 1, rt, bt),
                             (bt * rt, 0, 1, rt), c_size=mt * bt * rt)
    assert_close(orc, out, ref, nt * rt_l, what="seeded contraction")
