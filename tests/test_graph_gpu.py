"""Capturing the GEMM entry point into a CUDA graph (torch.cuda.graph) and replaying it.

Three launch kinds: an unsplit GEMM, a split-K GEMM reduced through distributed shared memory
(no workspace), and a split-K GEMM reduced through a global workspace (under capture its
counters are zeroed by a memset node instead of coming from the self-resetting ring, and its
workspace is a stream-ordered allocation inside the graph).  Each replay must give the eager
result bit for bit, twice in a row.
"""
import pytest

from gpu_util import options

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("MNK,opts", [((1024, 1024, 1024), {}),
                                      ((128, 4096, 8192), {}),
                                      ((128, 4096, 8192), {"cluster_fixup": 0})],
                         ids=["unsplit", "split_cluster", "split_global"])
def test_graph_capture_replays_eager_result(b2g, cuda, MNK, opts):
    torch = cuda
    M, N, K = MNK
    dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
    dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
    b2g.fill_uniform(dA, M * K, 81)
    b2g.fill_uniform(dB, K * N, 82)
    with options(b2g, **opts):
        eager = torch.empty((M, N), dtype=torch.float32, device="cuda")
        b2g.gemm(dA, dB, eager, M, N, K)
        torch.cuda.synchronize()
        dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up outside the capture (per-device set-up)
            b2g.gemm(dA, dB, dC, M, N, K, stream=side.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            b2g.gemm(dA, dB, dC, M, N, K, stream=torch.cuda.current_stream().cuda_stream)
        for _ in range(2):
            dC.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert b2g.device_status() == 0
            assert torch.equal(dC, eager)
        del g
