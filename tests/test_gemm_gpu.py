"""GPU parity tests of the GEMM entry points against the CPU oracle.

Reference semantics: GEMM_Naive, mmm.cpp:52-62 (C = A.B, fp32 accumulate, C overwritten).
Tolerance (written here, applied by oracle.orc.check):
    |C - R| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|R|   against the FP64 oracle R.
Inputs: seeded U[-1,1] fp16 (max|a| = max|b| = 1).
"""
import numpy as np
import pytest

from gpu_util import VARIANT_H_IDS, VARIANTS_H, assert_close, options, padded_f16, to_dev

pytestmark = pytest.mark.gpu


def _run_gemm(b2g, torch, orc, M, N, K, lda=None, ldb=None, ldc=None, seed=11):
    lda = lda or K
    ldb = ldb or N
    ldc = ldc or N
    A, dA = padded_f16(torch, orc, M, K, lda, seed)
    B, dB = padded_f16(torch, orc, K, N, ldb, seed + 1)
    dC = torch.full((max(M, 1), ldc), float("nan"), dtype=torch.float32, device="cuda")
    b2g.gemm(dA, dB, dC, M, N, K, lda, ldb, ldc)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    C = dC.cpu().numpy()[:M, :N]
    return A, B, C, b2g.last_path()


def test_fill_uniform_matches_oracle(b2g, cuda, orc):
    torch = cuda
    n = 1 << 20
    d = torch.empty(n, dtype=torch.float16, device="cuda")
    b2g.fill_uniform(d, n, 7, 12345)
    torch.cuda.synchronize()
    host = orc.uniform_f16((n,), 7, 12345)
    assert np.array_equal(d.cpu().numpy().view(np.uint16), host.view(np.uint16))


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
@pytest.mark.parametrize("MNK", [(128, 256, 64), (256, 256, 128), (512, 768, 320), (1024, 1024, 1024)])
def test_gemm_tile_multiples(b2g, cuda, orc, cg, tn, MNK):
    M, N, K = MNK
    with options(b2g, cta_group=cg, tile_n=tn):
        A, B, C, path = _run_gemm(b2g, cuda, orc, M, N, K)
    assert path == (b2g.PATH_TC_1CTA if cg == 1 else b2g.PATH_TC_2CTA)
    assert_close(orc, C, orc.gemm_f64(A, B), K, what="%s cg=%d" % (MNK, cg))


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
@pytest.mark.parametrize("MNK", [(1, 8, 8), (127, 129, 136), (129, 127, 1000), (1000, 1000, 8),
                                 (300, 40, 72), (8, 520, 64), (385, 264, 4104)])
def test_gemm_ragged_aligned_pitch(b2g, cuda, orc, cg, tn, MNK):
    """Ragged M/N/K (zero-filled loads, clipped stores) with 16-byte-aligned row pitches."""
    M, N, K = MNK
    r8 = lambda x: (x + 7) // 8 * 8
    with options(b2g, cta_group=cg, tile_n=tn):
        A, B, C, path = _run_gemm(b2g, cuda, orc, M, N, K, lda=r8(K), ldb=r8(N), ldc=r8(N) + 4)
    assert path in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    assert_close(orc, C, orc.gemm_f64(A, B), K, what="%s cg=%d" % (MNK, cg))


@pytest.mark.parametrize("MNK", [(127, 129, 127), (2, 3, 5), (33, 17, 50)])
def test_gemm_unaligned_runs_generic_bit_exact(b2g, cuda, orc, MNK):
    """Contiguous ragged shapes whose pitches break TMA's 16-byte rule: the generic kernel
    runs GEMM_Naive's exact arithmetic, so C equals the sequential fp32 oracle bit for bit."""
    M, N, K = MNK
    A, B, C, path = _run_gemm(b2g, cuda, orc, M, N, K)
    assert path == b2g.PATH_GENERIC
    ref = orc.gemm_f32_seq(A, B)
    assert np.array_equal(C.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("cg,tn", VARIANTS_H, ids=VARIANT_H_IDS)
def test_gemm_single_element(b2g, cuda, orc, cg, tn):
    """M = N = K = 1: every mode has extent 1, so the TMA path takes it (boxes larger than
    the tensor, zero-filled loads, clipped store)."""
    with options(b2g, cta_group=cg, tile_n=tn):
        A, B, C, path = _run_gemm(b2g, cuda, orc, 1, 1, 1)
    assert path in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    assert C[0, 0] == np.float32(A[0, 0]) * np.float32(B[0, 0])


def test_gemm_k0_zero_fill(b2g, cuda, orc):
    torch = cuda
    dC = torch.full((16, 16), 3.0, dtype=torch.float32, device="cuda")
    dA = torch.empty(16, dtype=torch.float16, device="cuda")
    b2g.gemm(dA, dA, dC, 16, 16, 0, 8, 16, 16)
    torch.cuda.synchronize()
    assert b2g.last_path() == b2g.PATH_ZERO
    assert float(dC.abs().max()) == 0.0


def test_gemm_known_answers(b2g, cuda, orc):
    """All-ones operands (C = K exactly) and B = identity (C = A exactly)."""
    torch = cuda
    M = N = K = 512
    ones = torch.ones((M, K), dtype=torch.float16, device="cuda")
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    b2g.gemm(ones, ones, C, M, N, K)
    torch.cuda.synchronize()
    assert bool((C == K).all())
    A = orc.uniform_f16((M, K), 5)
    eye = np.eye(K, dtype=np.float16)
    b2g.gemm(to_dev(torch, A), to_dev(torch, eye), C, M, N, K)
    torch.cuda.synchronize()
    assert np.array_equal(C.cpu().numpy(), A.astype(np.float32))
    # small integers: every product and partial sum is exact in fp32
    Ai = (np.arange(M * K) % 7 - 3).astype(np.float16).reshape(M, K)
    Bi = (np.arange(K * N) % 5 - 2).astype(np.float16).reshape(K, N)
    b2g.gemm(to_dev(torch, Ai), to_dev(torch, Bi), C, M, N, K)
    torch.cuda.synchronize()
    exact = Ai.astype(np.int64) @ Bi.astype(np.int64)
    assert np.array_equal(C.cpu().numpy().astype(np.int64), exact)


def test_gemm_reference_dropin_entry(b2g, cuda, orc):
    """b2g_gemm(A,B,C,M,N,K): the reference's contiguous, default-stream form."""
    torch = cuda
    M, N, K = 256, 512, 384
    A = orc.uniform_f16((M, K), 21)
    B = orc.uniform_f16((K, N), 22)
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    b2g.GEMM(to_dev(torch, A), to_dev(torch, B), C, M, N, K)
    torch.cuda.synchronize()
    assert_close(orc, C.cpu().numpy(), orc.gemm_f64(A, B), K)


def test_gemm_8192_sampled_rows(b2g, cuda, orc):
    """BASELINE configs[1] (8192^3): generated on the device with the oracle's generator,
    checked on a sample of rows (every 128-row tile and both halves of each CTA pair)."""
    torch = cuda
    M = N = K = 8192
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    b2g.fill_uniform(dA, M * K, 1)
    b2g.fill_uniform(dB, K * N, 2)
    b2g.gemm(dA, dB, dC, M, N, K)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    rows = sorted(set([0, 1, 127, 128, 255, 256, 4095, 4096, 8063, 8191] + list(range(37, M, 517))))
    A = orc.uniform_f16((M, K), 1)
    B = orc.uniform_f16((K, N), 2)
    sel = torch.tensor(rows, device="cuda")
    got = dC.index_select(0, sel).cpu().numpy()
    ref = np.concatenate([orc.gemm_f64(A, B, rows=(r, r + 1)) for r in rows])
    assert_close(orc, got, ref, K, what="8192^3 sampled rows")


def test_gemm_timeout_reports_error(b2g, cuda, orc):
    """Fault injection on the host side of the kernel: the producer issues no loads, the
    MMA's bounded wait runs out, the kernel records the code and returns; the context
    stays usable for the next call."""
    torch = cuda
    b2g.device_status(clear=True)
    M = N = K = 256
    dA = torch.zeros((M, K), dtype=torch.float16, device="cuda")
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    with options(b2g, fault_flags=1, timeout_ns=200_000_000, cta_group=1):
        b2g.gemm(dA, dA, dC, M, N, K)
        code = b2g.device_status(clear=True)
    assert code in (1, 2, 3, 4), code  # a wait of the producer, MMA or epilogue role gave up
    # the device still works
    A, B, C, path = _run_gemm(b2g, cuda, orc, 256, 256, 256)
    assert_close(orc, C, orc.gemm_f64(A, B), 256)


def test_gemm_c_larger_than_4gib(b2g, cuda, orc):
    """32768 x 32768 x 1024: C is 4 GiB (64-bit offsets everywhere).  Ternary operands first,
    where fp32 accumulation is exact in any order, so every element of C must equal the FP64
    product; then seeded U[-1,1] operands with rows near the start, middle and end checked
    against the FP64 oracle."""
    torch = cuda
    from test_fullsize_exact_gpu import _ternary, mismatches
    M = N = 32768
    K = 1024
    tA = _ternary(torch, (M, K), 41)
    tB = _ternary(torch, (K, N), 42)
    dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    b2g.gemm(tA, tB, dC, M, N, K)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert mismatches(torch, dC, tA, tB) == 0
    del tA, tB
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    b2g.fill_uniform(dA, M * K, 1)
    b2g.fill_uniform(dB, K * N, 2)
    b2g.gemm(dA, dB, dC, M, N, K)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    B = orc.uniform_f16((K, N), 2)
    for r in (0, 16383, 32767):
        a = orc.uniform_f16((1, K), 1, r * K)
        assert_close(orc, dC[r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K, what="row %d" % r)
    del dC
    torch.cuda.empty_cache()


def test_back_to_back_launches_with_and_without_pdl(b2g, cuda, orc):
    """Programmatic dependent launch (the default): each call of a chain C += A.B (beta = 1,
    the epilogue's TMA reduce-add reads C) depends on the C of the call just before it, launched
    right behind it.  The kernel waits on that dependency before it touches global memory, so
    the chain gives the same bits with and without PDL, and 5*A.B within tolerance."""
    torch = cuda
    M, N, K = 512, 768, 1024
    A = orc.uniform_f16((M, K), 31)
    B = orc.uniform_f16((K, N), 32)
    dA = torch.from_numpy(A.view(np.int16)).view(torch.float16).cuda()
    dB = torch.from_numpy(B.view(np.int16)).view(torch.float16).cuda()
    outs = {}
    for pdl in (1, 0):
        with options(b2g, pdl=pdl):
            dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
            b2g.gemm(dA, dB, dC, M, N, K)
            for _ in range(4):
                b2g.gemm_ex(dA, dB, dC, M, N, K, 1.0, 1.0)
            torch.cuda.synchronize()
            outs[pdl] = dC.clone()
    assert b2g.device_status() == 0
    assert torch.equal(outs[0], outs[1])
    assert_close(orc, outs[1].cpu().numpy(), 5.0 * orc.gemm_f64(A, B), K, 5.0, 1.0)


def test_launch_counter(b2g, cuda):
    """b2g_get_option("launches") counts the kernels the library launched (one per GEMM here)."""
    torch = cuda
    dA = torch.zeros((256, 512), dtype=torch.float16, device="cuda")
    dB = torch.zeros((512, 256), dtype=torch.float16, device="cuda")
    dC = torch.empty((256, 256), dtype=torch.float32, device="cuda")
    n0 = b2g.get_option("launches")
    for _ in range(5):
        b2g.gemm(dA, dB, dC, 256, 256, 512)
    torch.cuda.synchronize()
    assert b2g.get_option("launches") - n0 == 5

