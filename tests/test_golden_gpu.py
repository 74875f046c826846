"""GPU replay of the golden fixtures made by the reference's own code
(tests/golden/gen_golden.py).

* tensor-core path: within the tolerance |C - R| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|R|
  of the reference's GEMM_Naive output (row pitches padded to 16 bytes so TMA applies);
* generic path (forced): bit-identical to GEMM_Naive (same fp32 accumulation order);
* the reference's contraction (G[r][n][m][k] x In[b][n*rt_l+k] -> Out[m][b][r]) through
  b2g_contract5d_f16_f32 on the reference's strides, with no packing step.
"""
import os

import numpy as np
import pytest

from gpu_util import VARIANT_H_IDS, VARIANTS_H, assert_close, options, to_dev

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _cases():
    z = np.load(os.path.join(GOLDEN, "gemm_naive.npz"))
    return [(z["c%d_A" % i].view(np.float16), z["c%d_B" % i].view(np.float16), z["c%d_C" % i])
            for i in range(int(z["n_cases"]))]


def _padded(torch, X, ld):
    P = np.zeros((X.shape[0], ld), dtype=np.float16)
    P[:, :X.shape[1]] = X
    return to_dev(torch, P)


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
def test_golden_gemm_tensor_core_path(b2g, cuda, orc, cg, tn):
    torch = cuda
    r8 = lambda x: (x + 7) // 8 * 8
    for A, B, C in _cases():
        M, K = A.shape
        N = B.shape[1]
        lda, ldb, ldc = r8(K), r8(N), r8(N)
        dC = torch.full((M, ldc), float("nan"), dtype=torch.float32, device="cuda")
        with options(b2g, cta_group=cg, tile_n=tn):
            b2g.gemm(_padded(torch, A, lda), _padded(torch, B, ldb), dC, M, N, K, lda, ldb, ldc)
        torch.cuda.synchronize()
        assert b2g.last_path() in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
        max_a = float(np.abs(A.astype(np.float32)).max())
        max_b = float(np.abs(B.astype(np.float32)).max())
        assert_close(orc, dC.cpu().numpy()[:, :N], C.astype(np.float64), K, max_a, max_b,
                     what="golden %dx%dx%d" % (M, N, K))


def test_golden_gemm_generic_path_bit_exact(b2g, cuda, orc):
    torch = cuda
    for A, B, C in _cases():
        M, K = A.shape
        N = B.shape[1]
        dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
        with options(b2g, force_generic=1):
            b2g.gemm(to_dev(torch, A), to_dev(torch, B), dC, M, N, K)
        torch.cuda.synchronize()
        assert b2g.last_path() == b2g.PATH_GENERIC
        assert np.array_equal(dC.cpu().numpy().view(np.uint32), C.view(np.uint32))


def _ref_contraction(b2g, torch, force_generic):
    z = np.load(os.path.join(GOLDEN, "contraction_ref.npz"))
    mt, rt, nt, rt_l, bt = (int(x) for x in z["dims"])
    G = z["G"].view(np.float16)
    In = z["In"].view(np.float16)
    dOut = torch.full((mt * bt * rt,), float("nan"), dtype=torch.float32, device="cuda")
    with options(b2g, force_generic=force_generic):
        b2g.contract5d(to_dev(torch, G), (mt, 1, rt, nt, rt_l),
                       (rt_l, 0, nt * mt * rt_l, mt * rt_l, 1), to_dev(torch, In),
                       (nt, rt_l, bt), (rt_l, 1, nt * rt_l), dOut, (mt, 1, rt, bt),
                       (bt * rt, 0, 1, rt))
    torch.cuda.synchronize()
    return z, dOut.cpu().numpy(), b2g.last_path(), nt * rt_l


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
def test_golden_reference_contraction_tensor_core(b2g, cuda, orc, cg, tn):
    with options(b2g, cta_group=cg, tile_n=tn):
        z, out, path, K = _ref_contraction(b2g, cuda, 0)
    assert path in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    assert_close(orc, out, z["Out"].astype(np.float64), K, what="reference contraction")


def test_golden_reference_contraction_generic_bit_exact(b2g, cuda, orc):
    z, out, path, K = _ref_contraction(b2g, cuda, 1)
    assert path == b2g.PATH_GENERIC
    assert np.array_equal(out.view(np.uint32), z["Out"].view(np.uint32))
