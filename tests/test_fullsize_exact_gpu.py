"""Whole-matrix parity at BASELINE's full sizes, through an order-independent property.

With A and B drawn from {-1, 0, 1}, every product is -1, 0 or 1 and every partial sum an integer
of magnitude at most K < 2^24.  fp32 accumulation of such terms is exact in any order, so the
library's C must equal the FP64 product element for element on every path: CTA-pair tiles,
split-K with either fix-up, the contraction's 5-D tensor maps.  This checks every element of C
at the sizes BASELINE names, where the FP64 oracle could only afford sampled rows.  The FP64
product is torch's on the GPU, used here as the checker only.
"""
import pytest

from gpu_util import options

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ternary(torch, shape, seed):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    return torch.randint(-1, 2, shape, generator=g, device=DEV).to(torch.float16)


def mismatches(torch, C, A, B, block=4096):
    """Elements of C that differ from the FP64 product A.B, counted over row blocks (so the
    FP64 reference of a 32768 x 32768 C never exists whole)."""
    Bd = B.to(torch.float64)
    bad = 0
    for r0 in range(0, A.shape[0], block):
        ref = torch.mm(A[r0:r0 + block].to(torch.float64), Bd)
        bad += int((C[r0:r0 + block].to(torch.float64) != ref).sum().item())
        del ref
    return bad


def _exact_gemm(b2g, torch, M, N, K, seed):
    A = _ternary(torch, (M, K), seed)
    B = _ternary(torch, (K, N), seed + 1)
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=DEV)
    b2g.gemm(A, B, C, M, N, K)
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    return mismatches(torch, C, A, B)


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (8192, 8192, 8192), (16384, 16384, 4096),
                                   (8192, 28672, 8192)],
                         ids=["configs0", "configs1", "configs3_square", "configs3_wide"])
def test_gemm_full_size_exact(b2g, cuda, M, N, K):
    """BASELINE configs[0], [1] and the large configs[3] shapes, every element exact."""
    assert _exact_gemm(b2g, cuda, M, N, K, seed=M + N + K) == 0


@pytest.mark.parametrize("M,N,K", [(512, 512, 2048), (1024, 1024, 1024), (2048, 2048, 2048),
                                   (1024, 4096, 4096), (3072, 3072, 3072), (4096, 4096, 4096),
                                   (4096, 512, 1024)],
                         ids=["split4x8blocks", "configs0_split2", "pairs256_unsplit",
                              "pairs256_wide", "pairs512_72tiles", "pairs512_128tiles",
                              "n128_unsplit"])
def test_gemm_planner_small_and_mid_shapes_exact(b2g, cuda, M, N, K):
    """The plans the planner picks for small and mid-size shapes (one-CTA tiles split in 8-block
    pieces, unsplit 256x256 pair tiles, one or two waves of 512-wide pair tiles), every element
    exact."""
    assert _exact_gemm(b2g, cuda, M, N, K, seed=M * 3 + N * 5 + K) == 0


def test_gemm_32768_cubed_single_gpu_exact(b2g, cuda):
    """BASELINE configs[4]'s whole problem, 32768^3 (C is 4 GiB: 64-bit offsets in every
    address), on one GPU; every element exact."""
    torch = cuda
    assert _exact_gemm(b2g, torch, 32768, 32768, 32768, seed=11) == 0
    torch.cuda.empty_cache()


@pytest.mark.parametrize("cluster_fixup", [1, 0], ids=["cluster_fixup", "global_fixup"])
def test_gemm_skinny_full_size_exact(b2g, cuda, cluster_fixup):
    """BASELINE configs[3] 128 x 8192 x 8192: every tile split over K, reduced either through
    distributed shared memory or through the global workspace; every element exact."""
    with options(b2g, cluster_fixup=cluster_fixup):
        assert _exact_gemm(b2g, cuda, 128, 8192, 8192, seed=7) == 0


def test_contraction_full_size_exact(b2g, cuda):
    """C[a,b,i,n] = sum_{j,k} A[a,b,i,j,k] B[j,k,n] with a8 b16 i64 j64
    k128 n4096 through the contraction entry point; every element exact."""
    torch = cuda
    sa, sb, sc = (8, 16, 64, 64, 128), (64, 128, 4096), (8, 16, 64, 4096)

    def rowmajor(sh):
        st, acc = [], 1
        for d in reversed(sh):
            st.append(acc)
            acc *= d
        return tuple(reversed(st))

    A = _ternary(torch, sa, 21)
    B = _ternary(torch, sb, 22)
    C = torch.full(sc, float("nan"), dtype=torch.float32, device=DEV)
    b2g.contract5d(A, sa, rowmajor(sa), B, sb, rowmajor(sb), C, sc, rowmajor(sc))
    torch.cuda.synchronize()
    assert b2g.device_status() == 0
    ref = torch.mm(A.reshape(8 * 16 * 64, 64 * 128).to(torch.float64),
                   B.reshape(64 * 128, 4096).to(torch.float64)).reshape(sc)
    assert int((C.to(torch.float64) != ref).sum().item()) == 0


@pytest.mark.parametrize("M,N,K", [(8192, 8192, 8192), (8192, 28672, 8192), (8192, 4096, 8192)],
                         ids=["configs1", "configs3_wide", "configs2_view"])
@pytest.mark.parametrize("epi_warps", [4, 8])
def test_gemm_full_size_exact_epilogue_warps(b2g, cuda, M, N, K, epi_warps):
    """The 256 x 512 pair tile with four or eight epilogue warps (eight: each warp pulls 128
    columns of an N-half into registers before storing them); 8192 x 28672 x 8192 and the
    configs[2] GEMM view also split their tail wave over the global workspace.  Every element
    exact."""
    with options(b2g, epi_warps=epi_warps, tile_n=512):
        assert _exact_gemm(b2g, cuda, M, N, K, seed=M + N + K + epi_warps) == 0
