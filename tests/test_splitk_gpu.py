"""GPU tests of split-K (K split over several work units whose fp32 partial tiles are summed
in split order by the last unit of each tile) against the oracle.

Tolerance: |C - R| <= 1e-3*sqrt(K)*max|a|*max|b|*|alpha| + 1e-3*|R| against FP64.  Split-K is
deterministic: the partials of a tile are always summed in split order, so repeated calls give
identical bits (this also shows the per-tile counters are reset for the next call).
"""
import numpy as np
import pytest

from gpu_util import VARIANT_W8_IDS, VARIANTS_W8, assert_close, options, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cg,tn", VARIANTS_W8, ids=VARIANT_W8_IDS)
@pytest.mark.parametrize("splits", [2, 3, 5])
def test_split_k_forced(b2g, cuda, orc, cg, tn, splits):
    torch = cuda
    M, N, K = 384, 1024, 2048 + 192  # K blocks not divisible by the split count
    A = orc.uniform_f16((M, K), 61)
    B = orc.uniform_f16((K, N), 62)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    with options(b2g, cta_group=cg, tile_n=tn, split_k=splits):
        b2g.gemm(dA, dB, dC, M, N, K)
        torch.cuda.synchronize()
        assert b2g.device_status() == 0
        first = dC.clone()
        b2g.gemm(dA, dB, dC, M, N, K)
        torch.cuda.synchronize()
    assert torch.equal(first, dC)
    assert_close(orc, dC.cpu().numpy(), orc.gemm_f64(A, B), K, what="split %d" % splits)


def test_split_k_alpha_beta_and_ragged(b2g, cuda, orc):
    torch = cuda
    M, N, K = 200, 300, 1000
    r8 = lambda x: (x + 7) // 8 * 8
    A = orc.uniform_f16((M, K), 63)
    B = orc.uniform_f16((K, N), 64)
    C0 = orc.uniform_f16((M, N), 65).astype(np.float32)
    Ap = np.zeros((M, r8(K)), np.float16)
    Ap[:, :K] = A
    Bp = np.zeros((K, r8(N)), np.float16)
    Bp[:, :N] = B
    Cp = np.zeros((M, r8(N)), np.float32)
    Cp[:, :N] = C0
    dC = to_dev(torch, Cp)
    with options(b2g, split_k=4):
        b2g.gemm_ex(to_dev(torch, Ap), to_dev(torch, Bp), dC, M, N, K, 2.0, 1.0, lda=r8(K),
                    ldb=r8(N), ldc=r8(N))
    torch.cuda.synchronize()
    assert b2g.last_path() in (b2g.PATH_TC_1CTA, b2g.PATH_TC_2CTA)
    ref = 2.0 * orc.gemm_f64(A, B) + C0.astype(np.float64)
    assert_close(orc, dC.cpu().numpy()[:, :N], ref, K, 2.0, 1.0)


def test_split_k_reference_contraction(b2g, cuda, orc):
    """Split-K through the M-contiguous store of the reference's contraction layout."""
    torch = cuda
    mt, rt, nt, rt_l, bt = 4, 32, 16, 128, 256
    G = orc.uniform_f16((rt * nt * mt * rt_l,), 66)
    In = orc.uniform_f16((bt * nt * rt_l,), 67)
    a_shape, a_st = (mt, 1, rt, nt, rt_l), (rt_l, 0, nt * mt * rt_l, mt * rt_l, 1)
    b_shape, b_st = (nt, rt_l, bt), (rt_l, 1, nt * rt_l)
    c_shape, c_st = (mt, 1, rt, bt), (bt * rt, 0, 1, rt)
    dOut = torch.full((mt * bt * rt,), float("nan"), dtype=torch.float32, device="cuda")
    with options(b2g, split_k=3):
        b2g.contract5d(to_dev(torch, G), a_shape, a_st, to_dev(torch, In), b_shape, b_st, dOut,
                       c_shape, c_st)
    torch.cuda.synchronize()
    ref = orc.contract5d_f64(G, a_shape, a_st, In, b_shape, b_st, c_shape, c_st,
                             c_size=mt * bt * rt)
    assert_close(orc, dOut.cpu().numpy(), ref, nt * rt_l)


def test_split_k_auto_skinny(b2g, cuda, orc):
    """BASELINE configs[3]'s HBM-bound shape 128 x 8192 x 8192 takes split-K by default;
    checked on a sample of rows."""
    torch = cuda
    M, N, K = 128, 8192, 8192
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    b2g.fill_uniform(dA, M * K, 1)
    b2g.fill_uniform(dB, K * N, 2)
    b2g.gemm(dA, dB, dC, M, N, K)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    B = orc.uniform_f16((K, N), 2)
    for r in (0, 1, 63, 64, 127):
        a = orc.uniform_f16((1, K), 1, r * K)
        assert_close(orc, dC[r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K, what="row %d" % r)


@pytest.mark.parametrize("cg,tn", VARIANTS_W8, ids=VARIANT_W8_IDS)
def test_split_k_parallel_and_serial_fixup_agree(b2g, cuda, orc, cg, tn):
    """Both fix-up schedules sum the same partials in split order: identical bits."""
    torch = cuda
    M, N, K = 256, 1024, 4096
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(dA, M * K, 81)
    b2g.fill_uniform(dB, K * N, 82)
    outs = []
    for serial in (0, 1):
        dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        with options(b2g, cta_group=cg, tile_n=tn, split_k=4, serial_fixup=serial):
            b2g.gemm(dA, dB, dC, M, N, K)
        torch.cuda.synchronize()
        assert b2g.device_status() == 0
        outs.append(dC)
    assert torch.equal(outs[0], outs[1])
    A = orc.uniform_f16((M, K), 81)
    B = orc.uniform_f16((K, N), 82)
    assert_close(orc, outs[0].cpu().numpy(), orc.gemm_f64(A, B), K)


def test_tail_split_contraction_shape(b2g, cuda, orc):
    """8192 x 4096 x 8192 (BASELINE configs[2] as a GEMM view): 3.5 waves of 256x512 tiles,
    so only the tail wave's tiles are split in K.  Same result as without the tail split
    within tolerance, and correct against the oracle on sampled rows."""
    torch = cuda
    M, N, K = 8192, 4096, 8192
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(dA, M * K, 1)
    b2g.fill_uniform(dB, K * N, 2)
    res = {}
    for tail in (1, 0):
        dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        with options(b2g, tail_split=tail):
            b2g.gemm(dA, dB, dC, M, N, K)
        torch.cuda.synchronize()
        assert b2g.device_status() == 0
        res[tail] = dC
    diff = (res[1] - res[0]).abs().max().item()
    assert diff <= orc.tolerance(K, 1.0, 1.0), diff
    B = orc.uniform_f16((K, N), 2)
    for r in (0, 4095, 6000, 7935, 8191):
        a = orc.uniform_f16((1, K), 1, r * K)
        assert_close(orc, res[1][r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K, what="row %d" % r)


def test_split_k_counters_after_timeout_and_many_calls(b2g, cuda, orc):
    """Split-K arrival counters come from a per-device ring that every kernel leaves at zero.
    A split call whose waits run out (host-side fault injection: the producer issues no loads)
    is reported; clearing the error marks the ring for a full reset, and the following calls --
    many of them, each on a fresh range of the ring -- are correct and bit-identical."""
    torch = cuda
    b2g.device_status(clear=True)
    M, N, K = 256, 512, 4096
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(dA, M * K, 91)
    b2g.fill_uniform(dB, K * N, 92)
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    with options(b2g, fault_flags=1, timeout_ns=200_000_000, cta_group=1, tile_n=128, split_k=2):
        b2g.gemm(dA, dB, dC, M, N, K)
        code = b2g.device_status(clear=True)
    assert code in (1, 2, 3, 4, 6), code  # whichever bounded wait gave up first
    first = None
    with options(b2g, cta_group=1, tile_n=128, split_k=4):
        for _ in range(300):
            dC.fill_(float("nan"))
            b2g.gemm(dA, dB, dC, M, N, K)
            if first is None:
                torch.cuda.synchronize()
                first = dC.clone()
        torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert torch.equal(first, dC)
    A = orc.uniform_f16((M, K), 91)
    B = orc.uniform_f16((K, N), 92)
    assert_close(orc, dC.cpu().numpy(), orc.gemm_f64(A, B), K)


@pytest.mark.parametrize("tn,splits,MNK", [(128, 2, (128, 8192, 2048)), (256, 4, (128, 4096, 4096)),
                                           (128, 3, (200, 1000, 3000)), (256, 8, (256, 512, 8192)),
                                           (128, 5, (384, 1024, 2240))])
def test_cluster_fixup_matches_global_fixup(b2g, cuda, orc, tn, splits, MNK):
    """The cluster fix-up (partials reduced through distributed shared memory) and the global
    workspace fix-up sum the same partials in split order: identical bits, and correct."""
    torch = cuda
    M, N, K = MNK
    r8 = lambda x: (x + 7) // 8 * 8
    A = orc.uniform_f16((M, K), 71)
    B = orc.uniform_f16((K, N), 72)
    Ap = np.zeros((M, r8(K)), np.float16)
    Ap[:, :K] = A
    Bp = np.zeros((K, r8(N)), np.float16)
    Bp[:, :N] = B
    dA, dB = to_dev(torch, Ap), to_dev(torch, Bp)
    outs = []
    for cf in (1, 0):
        dC = torch.full((M, r8(N)), float("nan"), dtype=torch.float32, device="cuda")
        with options(b2g, cta_group=1, tile_n=tn, split_k=splits, cluster_fixup=cf):
            b2g.gemm(dA, dB, dC, M, N, K, lda=r8(K), ldb=r8(N), ldc=r8(N))
        torch.cuda.synchronize()
        assert b2g.device_status() == 0
        outs.append(dC[:, :N].clone())
    assert torch.equal(outs[0], outs[1])
    assert_close(orc, outs[0].cpu().numpy(), orc.gemm_f64(A, B), K)


def test_split_k_counter_ring_wraps_across_streams(b2g, cuda, orc):
    """Split calls on two streams share the per-device counter ring.  With the ring cut to 512
    slots (8 calls per lap) 64 calls alternate between the streams, so the ring wraps eight
    times while kernels of the other stream may still hold counters; every wrap first waits
    for the other stream's last user.  Every result must equal the single-stream result bit
    for bit, and no bounded wait may run out."""
    torch = cuda
    b2g.device_status(clear=True)
    M, N, K = 256, 1024, 4096
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(dA, M * K, 93)
    b2g.fill_uniform(dB, K * N, 94)
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    with options(b2g, cta_group=1, tile_n=128, split_k=4, cluster_fixup=0, ring_slots=512):
        ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
        b2g.gemm(dA, dB, ref, M, N, K)
        torch.cuda.synchronize()
        outs = [torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
                for _ in range(64)]
        torch.cuda.synchronize()
        for i, out in enumerate(outs):
            b2g.gemm(dA, dB, out, M, N, K, stream=streams[i % 2].cuda_stream)
        torch.cuda.synchronize()
    assert b2g.device_status() == 0
    for i, out in enumerate(outs):
        assert torch.equal(out, ref), i
    A = orc.uniform_f16((M, K), 93)
    B = orc.uniform_f16((K, N), 94)
    assert_close(orc, ref.cpu().numpy(), orc.gemm_f64(A, B), K)


@pytest.mark.parametrize("splits", [2, 3, 4])
@pytest.mark.parametrize("MNK", [(128, 1024, 4096), (100, 520, 3000), (256, 768, 2240),
                                 (64, 256, 8192)])
def test_half_pair_split_cluster_fixup(b2g, cuda, orc, splits, MNK):
    """Half-height pair tiles (128 x 256 over a CTA pair, 64 A rows per CTA) with K split 2-4
    ways: the splits of a tile are consecutive CTA pairs of one cluster, and each CTA sums its
    counterparts' partials (same rows, other splits) through distributed shared memory in
    split order.  Correct, and identical bits on a second call.  64 x 256 x 8192 leaves the
    second CTA of every pair without rows."""
    torch = cuda
    M, N, K = MNK
    r8 = lambda x: (x + 7) // 8 * 8
    A = orc.uniform_f16((M, K), 81)
    B = orc.uniform_f16((K, N), 82)
    Ap = np.zeros((M, r8(K)), np.float16)
    Ap[:, :K] = A
    Bp = np.zeros((K, r8(N)), np.float16)
    Bp[:, :N] = B
    dA, dB = to_dev(torch, Ap), to_dev(torch, Bp)
    outs = []
    with options(b2g, pair_rows=64, split_k=splits):
        for _ in range(2):
            dC = torch.full((M, r8(N)), float("nan"), dtype=torch.float32, device="cuda")
            b2g.gemm(dA, dB, dC, M, N, K, lda=r8(K), ldb=r8(N), ldc=r8(N))
            torch.cuda.synchronize()
            assert b2g.device_status() == 0
            assert b2g.last_path() == b2g.PATH_TC_2CTA
            assert b2g.get_option("last_split_ws_bytes") == 0  # no global workspace
            outs.append(dC[:, :N].clone())
    assert torch.equal(outs[0], outs[1])
    assert_close(orc, outs[0].cpu().numpy(), orc.gemm_f64(A, B), K, what="split %d" % splits)


def test_half_pair_refuses_a_split_it_cannot_reduce(b2g, cuda):
    """Forced half-height pair tiles split K only through the cluster fix-up (at most 4
    splits): a forced 5-way split, or the cluster fix-up turned off, is refused."""
    torch = cuda
    M, N, K = 128, 1024, 8192
    dA = torch.zeros((M, K), dtype=torch.float16, device="cuda")
    dB = torch.zeros((K, N), dtype=torch.float16, device="cuda")
    dC = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    for kw in (dict(split_k=5), dict(split_k=2, cluster_fixup=0)):
        with options(b2g, pair_rows=64, **kw):
            with pytest.raises(b2g.B2GError) as e:
                b2g.gemm(dA, dB, dC, M, N, K)
        assert e.value.code == b2g.ERR_UNSUPPORTED


def test_skinny_half_pairs_agree_with_the_default_plan(b2g, cuda, orc):
    """BASELINE configs[3] 128 x 8192 x 8192: forced half-height pair tiles (K split 2 ways)
    agree with the default plan (one-CTA tiles, K split 4 ways) within tolerance, and both
    with the oracle on sampled rows."""
    torch = cuda
    M, N, K = 128, 8192, 8192
    assert b2g.plan_preview(M, N, K, rows=True) == (1, 256, 4, 0, 128)
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(dA, M * K, 83)
    b2g.fill_uniform(dB, K * N, 84)
    res = {}
    for rows in (0, 64):
        with options(b2g, pair_rows=rows):
            dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
            b2g.gemm(dA, dB, dC, M, N, K)
            torch.cuda.synchronize()
            assert b2g.device_status() == 0
            res[rows] = dC
    assert_close(orc, res[64].cpu().numpy(), res[0].cpu().numpy().astype(np.float64), K)
    B = orc.uniform_f16((K, N), 84)
    for r in (0, 31, 32, 63, 64, 100, 127):
        a = orc.uniform_f16((1, K), 83, r * K)
        for rows in (0, 64):
            assert_close(orc, res[rows][r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K,
                         what="row %d pair_rows %d" % (r, rows))
