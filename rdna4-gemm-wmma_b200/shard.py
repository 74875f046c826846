"""Sharding of C = A.B across ranks of a torch.distributed process group: the pipelines of the
C entry points in csrc/b2g_shard.cu, driven through torch.distributed for callers that already
run one process per GPU under torchrun.

* sharded_gemm (b2g_gemm_sharded), M-row slabs: B is broadcast from `root` in K-row panels
  and each rank multiplies its own row slab of A by each panel as it arrives (panel 0
  overwrites the C slab, later panels add into it).  C stays local: no reduction, no gather.
* sharded_gemm_k (b2g_gemm_sharded_k), K slabs: each rank multiplies its K slab of A and B
  into an fp32 partial of the whole C; a reduce-scatter leaves each rank M/world summed rows.
* sharded_gemm_n (b2g_gemm_sharded_n), N slabs: A is broadcast from `root` in row panels,
  each rank computes its column slab of C; an optional all-gather assembles the whole C.

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


def sharded_gemm_k(A_kslab, B_kslab, C_slab, M, N, K, group=None, gemm=None):
    """K-split + reduce-scatter.  A_kslab: M x k_r, B_kslab: k_r x N with (k0, k_r) =
    slab_rows(K, world, rank); C_slab: M/world x N receives rows [rank*M/world, ...) of C.
    The partial is fp32 (as in the C library) unless C_slab has another type."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if M % world:
        raise ValueError("M must be a multiple of the rank count")
    k0, kr = slab_rows(K, world, rank)
    rows = M // world
    gemm = gemm or _b2g_gemm
    P = torch.empty((M, N), dtype=C_slab.dtype, device=C_slab.device)
    gemm(A_kslab, B_kslab, P, M, N, kr, 0.0, A_kslab.stride(0) if kr else 1, B_kslab.stride(0),
         N)
    out = C_slab if C_slab.is_contiguous() else torch.empty((rows, N), dtype=C_slab.dtype,
                                                             device=C_slab.device)
    dist.reduce_scatter_tensor(out, P, group=group)
    if out is not C_slab:
        C_slab.copy_(out)
    return rank * rows, rows


class PeerFailedError(RuntimeError):
    """A peer's part of a collective call failed, so this rank's result is invalid (it has been
    filled with NaN)."""


def sharded_gemm_k_p2p(A_kslab, B_kslab, C_slab, M, N, K, group=None, gemm=None):
    """The schedule of b2g_gemm_sharded_k_p2p.  This rank computes its partial one row slab at a
    time, the other ranks' slabs first (q = rank+1, ..., rank-1) and its own last; slab q lands
    in receive slot `rank` of rank q; every rank sums its slots in rank order (slot 0 first).
    The C library stores each slab into the owner's slot over peer memory from the GEMM's
    epilogue; here each slab travels as one point-to-point message.  Returns (row0, rows).

    Failure: a rank whose own arguments are invalid (here a C_slab narrower than N, the
    library's ldc < N) still takes every step of the protocol but skips its GEMMs, and tells
    the others so (the library writes a status word into every peer's flags before its
    'landed' flag; here the statuses are all-gathered).  It raises ValueError; every other rank
    fills its C_slab with NaN and raises PeerFailedError (the library reports that through the
    device error word, b2g_device_status)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if M % world:
        raise ValueError("M must be a multiple of the rank count")
    k0, kr = slab_rows(K, world, rank)
    rows = M // world
    ok = C_slab.dim() == 2 and C_slab.shape[0] >= rows and C_slab.shape[1] >= N
    gemm = gemm or _b2g_gemm
    peer = (lambda q: dist.get_global_rank(group, q)) if group is not None else (lambda q: q)
    slots = torch.zeros((world, rows, N), dtype=C_slab.dtype, device=C_slab.device)
    lda = A_kslab.stride(0) if kr else 1
    reqs, parts = [], []
    for t in range(1, world + 1):
        q = (rank + t) % world
        part = slots[rank] if q == rank else torch.zeros((rows, N), dtype=slots.dtype,
                                                          device=C_slab.device)
        if ok:
            gemm(A_kslab[q * rows:(q + 1) * rows], B_kslab, part, rows, N, kr, 0.0, lda,
                 B_kslab.stride(0), N)
        if q != rank:
            parts.append(part)
            reqs.append(dist.isend(part, peer(q), group=group))
    for q in range(world):
        if q != rank:
            reqs.append(dist.irecv(slots[q], peer(q), group=group))
    status = torch.tensor([0 if ok else 1], dtype=torch.int32)
    statuses = [torch.zeros(1, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(statuses, status, group=group)
    for r in reqs:
        r.wait()
    if not ok:
        raise ValueError("C_slab must hold M/world rows of N columns")
    failed = [q for q in range(world) if q != rank and int(statuses[q].item())]
    if failed:
        C_slab[:rows, :N] = float("nan")
        raise PeerFailedError("the part of rank(s) %s failed" % failed)
    acc = slots[0].clone()
    for q in range(1, world):
        acc += slots[q]
    C_slab.copy_(acc)
    return rank * rows, rows


def sharded_gemm_n(A, B_nslab, C_nslab, M, N, K, group=None, root=0, panels=4, C_full=None,
                   gemm=None):
    """N slabs: A (M x K on every rank, filled from `root`) arrives in row panels (multiples of
    64 rows but the last), each followed by the GEMM of its rows against this rank's column
    slab B_nslab (K x n_r, (n0, n_r) = slab_rows(N, world, rank)) into C_nslab (M x n_r).
    With C_full (M x N, N a multiple of world) every rank also receives the whole C."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n0, nr = slab_rows(N, world, rank)
    gemm = gemm or _b2g_gemm
    src = dist.get_global_rank(group, root) if group else root
    for m0, m1 in k_panels(M, panels):
        if m1 > m0:
            dist.broadcast(A[m0:m1], src=src, group=group)
            if nr > 0:
                gemm(A[m0:], B_nslab, C_nslab[m0:], m1 - m0, nr, K, 0.0, A.stride(0),
                     B_nslab.stride(0), C_nslab.stride(0))
    if C_full is not None:
        if N % world:
            raise ValueError("the gathered C needs N to be a multiple of the rank count")
        nw = N // world
        G = torch.empty((world * M, nw), dtype=C_nslab.dtype, device=C_nslab.device)
        dist.all_gather_into_tensor(G, C_nslab[:M, :nw].contiguous(), group=group)
        C_full.copy_(G.view(world, M, nw).permute(1, 0, 2).reshape(M, N))
    return n0, nr
