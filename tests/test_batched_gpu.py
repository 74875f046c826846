"""GPU tests of batch modes (b2g_gemm_batched, b2g_contract5d_batched) against the FP64 oracle.

Mode a of the contraction becomes a batch mode shared by B: C[a,b,i,n] = sum_{j,k}
A[a,b,i,j,k] B[a,j,k,n].  A tile never spans two batch entries, so per-batch row counts below
the 128-row tile are zero-filled on load and clipped on store; each batch entry is checked
against its own oracle product.  Tolerance: |C - R| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|R|.
"""
import numpy as np
import pytest

from gpu_util import assert_close, options, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("opts", [{}, {"tile_n": 128}, {"tile_n": 256, "split_k": 3},
                                  {"tile_n": 128, "split_k": 2, "cluster_fixup": 0}],
                         ids=["auto", "n128", "n256_split3", "n128_split2_global"])
def test_gemm_batched(b2g, cuda, orc, opts):
    torch = cuda
    L, M, N, K = 3, 200, 300, 640
    lda, ldb, ldc = 648, 304, 304
    sa, sb, sc = M * lda + 64, K * ldb + 64, M * ldc + 64
    A = orc.uniform_f16((L * sa,), 11)
    B = orc.uniform_f16((L * sb,), 12)
    dC = torch.full((L * sc,), float("nan"), dtype=torch.float32, device="cuda")
    with options(b2g, **opts):
        b2g.gemm_batched(to_dev(torch, A), to_dev(torch, B), dC, L, M, N, K, sa, sb, sc,
                         lda=lda, ldb=ldb, ldc=ldc)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert b2g.last_path() in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)  # 2 M tiles per batch: pairs allowed
    C = dC.cpu().numpy()
    for l in range(L):
        Al = A[l * sa: l * sa + M * lda].reshape(M, lda)[:, :K]
        Bl = B[l * sb: l * sb + K * ldb].reshape(K, ldb)[:, :N]
        Cl = C[l * sc: l * sc + M * ldc].reshape(M, ldc)
        assert_close(orc, Cl[:, :N], orc.gemm_f64(Al, Bl), K, what="batch %d %r" % (l, opts))
        assert np.isnan(Cl[:, N:]).all()
    assert np.isnan(C[M * ldc: sc]).all()  # gap between batches untouched


def test_gemm_batched_generic(b2g, cuda, orc):
    torch = cuda
    L, M, N, K = 2, 21, 13, 37  # unaligned pitches: the generic kernel
    A = orc.uniform_f16((L, M, K), 13)
    B = orc.uniform_f16((L, K, N), 14)
    dC = torch.empty((L, M, N), dtype=torch.float32, device="cuda")
    b2g.gemm_batched(to_dev(torch, A), to_dev(torch, B), dC, L, M, N, K, M * K, K * N, M * N)
    torch.cuda.synchronize()
    assert b2g.last_path() == b2g.PATH_GENERIC
    for l in range(L):
        assert_close(orc, dC[l].cpu().numpy(), orc.gemm_f64(A[l], B[l]), K)


@pytest.mark.parametrize("shape", [(4, 3, 16, 2, 64, 256), (2, 2, 64, 4, 64, 512),
                                   (3, 1, 200, 1, 128, 264)])
def test_contraction_batched(b2g, cuda, orc, shape):
    torch = cuda
    a, b, i, j, k, n = shape
    st = lambda sh: [int(np.prod(sh[d + 1:])) for d in range(len(sh))]
    A = orc.uniform_f16((a * b * i * j * k,), 15)
    B = orc.uniform_f16((a * j * k * n,), 16)
    dC = torch.full((a * b * i * n,), float("nan"), dtype=torch.float32, device="cuda")
    b2g.contract5d_batched(to_dev(torch, A), (a, b, i, j, k), st((a, b, i, j, k)), to_dev(torch, B),
                           (j, k, n), st((j, k, n)), j * k * n, dC, (a, b, i, n),
                           st((a, b, i, n)))
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert b2g.last_path() in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)  # 2 M tiles per batch: pairs allowed
    C = dC.cpu().numpy().reshape(a, b * i, n)
    A4 = A.reshape(a, b * i, j * k)
    B4 = B.reshape(a, j * k, n)
    for l in range(a):
        assert_close(orc, C[l], orc.gemm_f64(A4[l], B4[l]), j * k, what="batch %d %r" % (l, shape))


@pytest.mark.parametrize("M", [2048, 2176])
def test_gemm_batched_large(b2g, cuda, orc, M):
    """Large batch entries: CTA-pair tiles when the M tiles per batch entry are even (2048 rows
    = 16 tiles), one-CTA tiles when odd (2176 rows = 17 tiles); rows sampled per batch."""
    torch = cuda
    L, N, K = 3, 2048, 1024
    dA = torch.empty((L, M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((L, K, N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(dA, L * M * K, 21)
    b2g.fill_uniform(dB, L * K * N, 22)
    dC = torch.empty((L, M, N), dtype=torch.float32, device="cuda")
    b2g.gemm_batched(dA, dB, dC, L, M, N, K, M * K, K * N, M * N)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert b2g.last_path() == (b2g.PATH_TC_2CTA if M % 256 == 0 else b2g.PATH_TC_1CTA)
    for l in range(L):
        B = orc.uniform_f16((K * N,), 22, l * K * N).reshape(K, N)
        for r in (0, 127, 128, M // 2, M - 1):
            a = orc.uniform_f16((1, K), 21, (l * M + r) * K)
            assert_close(orc, dC[l, r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K,
                         what="batch %d row %d" % (l, r))
