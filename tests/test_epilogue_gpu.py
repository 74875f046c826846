"""GPU tests of the alpha/beta epilogue (b2g_gemm_ex, b2g_contract5d_ex) against the oracle.

C = alpha*A.B + beta*C.  beta = 0 must not read C (a NaN-filled C stays out of the result),
beta = 1 adds through the TMA reduce-add epilogue, other beta values scale C first.
Tolerance: |C - R| <= 1e-3*sqrt(K)*max|a|*max|b|*|alpha| + 1e-3*|R| (+ the rounding of the
beta*C term, far below it) against an FP64 reference R.
"""
import numpy as np
import pytest

from gpu_util import VARIANT_H_IDS, VARIANTS_H, assert_close, options, to_dev

pytestmark = pytest.mark.gpu


def _inputs(orc, M, N, K, seed=31):
    return orc.uniform_f16((M, K), seed), orc.uniform_f16((K, N), seed + 1), \
        orc.uniform_f16((M, N), seed + 2).astype(np.float32)


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
@pytest.mark.parametrize("alpha,beta", [(2.0, 0.0), (1.0, 1.0), (-0.5, 1.0), (1.5, 0.25)])
def test_gemm_alpha_beta(b2g, cuda, orc, cg, tn, alpha, beta):
    torch = cuda
    M, N, K = 384, 640, 320
    A, B, C0 = _inputs(orc, M, N, K)
    dC = to_dev(torch, C0 if beta != 0.0 else np.full_like(C0, np.nan))
    with options(b2g, cta_group=cg, tile_n=tn):
        b2g.gemm_ex(to_dev(torch, A), to_dev(torch, B), dC, M, N, K, alpha, beta)
    torch.cuda.synchronize()
    assert b2g.last_path() in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    ref = alpha * orc.gemm_f64(A, B) + (beta * C0.astype(np.float64) if beta else 0.0)
    assert_close(orc, dC.cpu().numpy(), ref, K, abs(alpha), 1.0, what="alpha=%g beta=%g" % (alpha, beta))


@pytest.mark.parametrize("alpha,beta", [(2.0, 0.0), (1.0, 1.0), (1.5, 0.25)])
def test_gemm_alpha_beta_generic(b2g, cuda, orc, alpha, beta):
    torch = cuda
    M, N, K = 33, 17, 50  # unaligned pitches: generic kernel
    A, B, C0 = _inputs(orc, M, N, K)
    dC = to_dev(torch, C0 if beta != 0.0 else np.full_like(C0, np.nan))
    b2g.gemm_ex(to_dev(torch, A), to_dev(torch, B), dC, M, N, K, alpha, beta)
    torch.cuda.synchronize()
    assert b2g.last_path() == b2g.PATH_GENERIC
    ref = alpha * orc.gemm_f64(A, B) + (beta * C0.astype(np.float64) if beta else 0.0)
    assert_close(orc, dC.cpu().numpy(), ref, K, abs(alpha), 1.0)


def test_gemm_k_panels_accumulate(b2g, cuda, orc):
    """C = A.B computed as four K panels (the first overwrites, the rest add with beta = 1):
    the pattern the sharded path uses while B is still arriving."""
    torch = cuda
    M, N, K = 512, 1024, 1024
    A, B, _ = _inputs(orc, M, N, K, seed=41)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    P = 4
    kp = K // P
    for p in range(P):
        b2g.gemm_ex(dA[:, p * kp:], dB[p * kp:], dC, M, N, kp, 1.0, 0.0 if p == 0 else 1.0,
                    lda=K, ldb=N, ldc=N)
    torch.cuda.synchronize()
    assert_close(orc, dC.cpu().numpy(), orc.gemm_f64(A, B), K)
    # deterministic: the same sequence gives the same bits
    first = dC.clone()
    for p in range(P):
        b2g.gemm_ex(dA[:, p * kp:], dB[p * kp:], dC, M, N, kp, 1.0, 0.0 if p == 0 else 1.0,
                    lda=K, ldb=N, ldc=N)
    torch.cuda.synchronize()
    assert torch.equal(first, dC)


def test_gemm_k0_beta(b2g, cuda, orc):
    """K == 0: C = beta*C (beta = 1 leaves C untouched, beta = 0 zeroes it)."""
    torch = cuda
    C0 = orc.uniform_f16((16, 16), 3).astype(np.float32)
    dA = torch.empty(16, dtype=torch.float16, device="cuda")
    for beta in (0.0, 1.0, 3.0):
        dC = to_dev(torch, C0)
        b2g.gemm_ex(dA, dA, dC, 16, 16, 0, 1.0, beta, lda=8)
        torch.cuda.synchronize()
        assert np.array_equal(dC.cpu().numpy(), (C0 * np.float32(beta)).astype(np.float32))


def test_contract_reference_form_accumulate(b2g, cuda, orc):
    """beta = 1 through the M-contiguous (transposed) store of the reference contraction."""
    torch = cuda
    mt, rt, nt, rt_l, bt = 8, 32, 2, 64, 256
    G = orc.uniform_f16((rt * nt * mt * rt_l,), 51)
    In = orc.uniform_f16((bt * nt * rt_l,), 52)
    C0 = orc.uniform_f16((mt * bt * rt,), 53).astype(np.float32)
    a_shape, a_st = (mt, 1, rt, nt, rt_l), (rt_l, 0, nt * mt * rt_l, mt * rt_l, 1)
    b_shape, b_st = (nt, rt_l, bt), (rt_l, 1, nt * rt_l)
    c_shape, c_st = (mt, 1, rt, bt), (bt * rt, 0, 1, rt)
    dC = to_dev(torch, C0)
    b2g.contract5d_ex(to_dev(torch, G), a_shape, a_st, to_dev(torch, In), b_shape, b_st, dC,
                      c_shape, c_st, 1.0, 1.0)
    torch.cuda.synchronize()
    assert b2g.last_path() in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    ref = orc.contract5d_f64(G, a_shape, a_st, In, b_shape, b_st, c_shape, c_st,
                             c_size=mt * bt * rt) + C0.astype(np.float64)
    assert_close(orc, dC.cpu().numpy(), ref, nt * rt_l)
