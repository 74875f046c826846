"""M-row-slab sharding of C = A.B across ranks of a torch.distributed process group.

The same pipeline as the C entry point b2g_gemm_sharded (csrc/b2g_shard.cu), driven through
torch.distributed for callers that already run one process per GPU under torchrun: B is
broadcast from `root` in K-row panels and each rank multiplies its own row slab of A by each
panel as it arrives (panel 0 overwrites the C slab, later panels add into it).  C stays
local: no reduction, no gather.

`gemm(A_view, B_view, C, rows, N, k, beta)` is the per-panel compute.  It defaults to the CUDA
library (b2g_gemm_ex); host-side tests pass a CPU stand-in to check the partition and the
panel schedule on gloo ranks without a GPU.
"""


def slab_rows(M, world, rank):
    """Balanced contiguous partition: M // world rows each, the first M % world ranks one more
    (the rule of b2g_slab_rows)."""
    base, rem = divmod(M, world)
    rows = base + (1 if rank < rem else 0)
    return rank * base + min(rank, rem), rows


def k_panels(K, panels, align=64):
    """[(k0, k1)] panel bounds: multiples of `align` except possibly the last."""
    panels = max(1, int(panels))
    if K <= 0:
        return [(0, 0)]
    kp = -(-K // panels)
    kp = -(-kp // align) * align
    return [(k0, min(K, k0 + kp)) for k0 in range(0, K, kp)]


def _b2g_gemm(A_view, B_view, C, rows, N, k, beta, lda, ldb, ldc):
    import importlib.util
    import os
    import sys
    if "b2g" not in sys.modules:
        here = os.path.dirname(os.path.abspath(__file__))
        spec = importlib.util.spec_from_file_location("b2g", os.path.join(here, "b2g.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules["b2g"] = mod
        spec.loader.exec_module(mod)
    sys.modules["b2g"].gemm_ex(A_view, B_view, C, rows, N, k, 1.0, beta, lda=lda, ldb=ldb, ldc=ldc)


def sharded_gemm(A_slab, B, C_slab, M, N, K, group=None, root=0, panels=4, gemm=None):
    """This rank's part of C = A.B.  A_slab: this rank's rows of A (rows x K), B: K x N on every
    rank (filled from `root`), C_slab: rows x N.  Returns (row0, rows)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    row0, rows = slab_rows(M, world, rank)
    assert A_slab.shape[0] >= rows and C_slab.shape[0] >= rows
    gemm = gemm or _b2g_gemm
    for p, (k0, k1) in enumerate(k_panels(K, panels)):
        if k1 > k0:
            panel = B[k0:k1]
            dist.broadcast(panel, src=dist.get_global_rank(group, root) if group else root,
                           group=group)
        if rows > 0:
            gemm(A_slab[:, k0:], B[k0:], C_slab, rows, N, k1 - k0, 0.0 if p == 0 else 1.0,
                 A_slab.stride(0), B.stride(0), C_slab.stride(0))
    return row0, rows
