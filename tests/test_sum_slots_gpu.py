"""b2g_gemm_sum_slots: C = the sum, in slot order, of A.B (slot `self`) and fp32 slots.

The property checked is bit equality with the unfused computation: b2g_gemm_f16_f32 into a
buffer, then the terms added in order s = 0, 1, ... (fp32 addition is exactly defined, so the
same order gives the same bits).  The A.B term itself is checked against the FP64 oracle on
sampled rows.  Shapes cover the tensor-core epilogue (whole and partial tiles, split-K) and the
separate pass (rows not 16-byte aligned, K = 0)."""
import pytest

from gpu_util import options

pytestmark = pytest.mark.gpu


def _unfused(b2g, torch, A, B, slots, M, N, K, count, self_index):
    P = torch.empty((M, N), dtype=torch.float32, device="cuda")
    b2g.gemm(A, B, P, M, N, K, lda=max(K, 1))
    acc = None
    for s in range(count):
        t = P if s == self_index else slots[s]
        acc = t.clone() if acc is None else acc + t
    return acc


def _inputs(b2g, torch, M, N, K, count, seed):
    A = torch.empty((M, max(K, 1)), dtype=torch.float16, device="cuda")
    B = torch.empty((max(K, 1), N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(A, A.numel(), seed)
    b2g.fill_uniform(B, B.numel(), seed + 1)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed + 2)
    slots = torch.empty((count, M, N), dtype=torch.float32, device="cuda")
    slots.uniform_(-300.0, 300.0, generator=g)  # partials of other ranks: larger than A.B
    return A, B, slots


@pytest.mark.parametrize("M,N,K", [(4096, 8192, 4096), (520, 1000, 784), (128, 8192, 8192),
                                   (100, 1001, 300), (64, 256, 0)],
                         ids=["pair_tiles", "partial_tiles", "split_k", "separate_pass", "k0"])
@pytest.mark.parametrize("count,self_index", [(1, 0), (2, 0), (2, 1), (4, 2), (8, 7)])
def test_sum_slots_matches_unfused(b2g, cuda, M, N, K, count, self_index):
    torch = cuda
    A, B, slots = _inputs(b2g, torch, M, N, K, count, seed=M + N + K + count)
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    b2g.gemm_sum_slots(A, B, C, M, N, K, slots, M * N, count, self_index, lda=max(K, 1))
    ref = _unfused(b2g, torch, A, B, slots, M, N, K, count, self_index)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert torch.equal(C.view(torch.int32), ref.view(torch.int32))


@pytest.mark.parametrize("epi_warps", [4, 8])
def test_sum_slots_pair_tile_epilogue_warps_and_padded_c(b2g, cuda, epi_warps):
    """The 256 x 512 pair tile with four and eight epilogue warps, C with a padded pitch (the
    pad is left alone) and slots further apart than M * N."""
    torch = cuda
    M, N, K, count = 2048, 4096, 2048, 3
    A, B, _ = _inputs(b2g, torch, M, N, K, count, seed=5)
    stride = M * N + 64
    flat = torch.empty((count * stride,), dtype=torch.float32, device="cuda").uniform_(-50, 50)
    slots = [flat[s * stride:s * stride + M * N].view(M, N) for s in range(count)]
    C = torch.full((M, N + 4), float("nan"), dtype=torch.float32, device="cuda")
    with options(b2g, tile_n=512, cta_group=2, epi_warps=epi_warps):
        b2g.gemm_sum_slots(A, B, C, M, N, K, flat, stride, count, 1, ldc=N + 4)
        ref = _unfused(b2g, torch, A, B, slots, M, N, K, count, 1)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert torch.equal(C[:, :N].contiguous().view(torch.int32), ref.view(torch.int32))
    assert bool(torch.isnan(C[:, N:]).all())


def test_sum_slots_term_is_the_oracle_product(b2g, cuda):
    """With every other slot zero, C is A.B: sampled rows against the FP64 oracle."""
    torch = cuda
    from oracle import orc
    M, N, K = 1024, 2048, 1536
    A = torch.empty((M, K), dtype=torch.float16, device="cuda")
    B = torch.empty((K, N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(A, M * K, 41)
    b2g.fill_uniform(B, K * N, 42)
    slots = torch.zeros((3, M, N), dtype=torch.float32, device="cuda")
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    b2g.gemm_sum_slots(A, B, C, M, N, K, slots, M * N, 3, 2)
    torch.cuda.synchronize()
    Bh = orc.uniform_f16((K, N), 42)
    bad = 0
    for r in (0, 1, 511, 1023):
        a = orc.uniform_f16((1, K), 41, r * K)
        bad += orc.check(C[r:r + 1].cpu().numpy(), orc.gemm_f64(a, Bh), K, 1.0, 1.0)[0]
    assert bad == 0


@pytest.mark.parametrize("M,N,K", [(1024, 2048, 1024), (100, 1001, 300)],
                         ids=["epilogue", "separate_pass"])
def test_sum_slots_failed_status_gives_nan_and_status_7(b2g, cuda, M, N, K):
    """A status word that is not the epoch (a peer whose part failed): C is NaN everywhere and
    the device error word reads 7; with every word at the epoch the sum is stored."""
    torch = cuda
    A, B, slots = _inputs(b2g, torch, M, N, K, 3, seed=9)
    status = torch.tensor([5, 5, 5], dtype=torch.int32, device="cuda")
    C = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    b2g.gemm_sum_slots(A, B, C, M, N, K, slots, M * N, 3, 0, status=status, epoch=5)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    assert not bool(torch.isnan(C).any())
    status[2] = 5 | (1 << 30)
    b2g.gemm_sum_slots(A, B, C, M, N, K, slots, M * N, 3, 0, status=status, epoch=5)
    torch.cuda.synchronize()
    assert b2g.device_status() == 7  # read and cleared
    assert bool(torch.isnan(C).all())
    assert b2g.device_status() == 0
