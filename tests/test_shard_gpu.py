"""GPU tests of b2g_gemm_sharded (M-row slabs, B broadcast from rank 0 in K panels over NCCL,
panel GEMMs accumulating into the local C slab) against the oracle.

* one rank on one GPU (a one-rank NCCL communicator): the whole pipeline -- communicator,
  panel broadcasts on the internal stream, event ordering, panel accumulation -- runs;
* two ranks on two GPUs (skipped with fewer): each rank's slab rows checked, and B on the
  non-root rank (filled with NaN before the call) must equal the root's bit for bit.
The tensor-parallel variants b2g_gemm_sharded_k (K slabs, fp32 partials reduce-scattered into
M/world-row slabs) and b2g_gemm_sharded_n (N slabs, A broadcast in row panels, optional
all-gather of C) run the same way: one rank in-process, two ranks as spawned processes.
Tolerance: |C - R| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|R| against the FP64 oracle.
"""
import multiprocessing as mp
import os
import sys
import tempfile

import numpy as np
import pytest

from gpu_util import assert_close

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import shard_worker  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,panels", [(1024, 1536, 2048, 4), (640, 512, 200, 3)])
def test_sharded_single_rank(b2g, cuda, orc, M, N, K, panels):
    torch = cuda
    uid = b2g.comm_unique_id()
    comm = b2g.comm_init(1, 0, uid)
    try:
        dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
        dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dA, M * K, 1)
        b2g.fill_uniform(dB, K * N, 2)
        dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        b2g.gemm_sharded(dA, dB, dC, M, N, K, comm, root=0, k_panels=panels)
        torch.cuda.synchronize()
        assert b2g.device_status() == 0
        A = orc.uniform_f16((M, K), 1)
        B = orc.uniform_f16((K, N), 2)
        assert_close(orc, dC.cpu().numpy(), orc.gemm_f64(A, B), K)
        assert np.array_equal(dB.cpu().numpy().view(np.uint16), B.view(np.uint16))
    finally:
        b2g.comm_destroy(comm)


def test_sharded_two_ranks(b2g, cuda):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        uid_path = os.path.join(d, "nccl_id")
        M, N, K = 4096, 2048, 4096
        procs = [ctx.Process(target=shard_worker.nccl_sharded_rank,
                             args=(r, 2, uid_path, M, N, K, 4, q)) for r in range(2)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    for rank, rows, worst, status, b_ok, tb in res:
        assert tb is None, tb
        assert status == 0 and worst == 0 and b_ok, (rank, rows, worst, status, b_ok)
    assert sum(r[1] for r in res) == M


class _ListQueue(list):
    put = list.append


@pytest.mark.parametrize("mode", ["k", "n"])
def test_tp_single_rank(b2g, cuda, mode):
    with tempfile.TemporaryDirectory() as d:
        q = _ListQueue()
        shard_worker.nccl_tp_rank(mode, 0, 1, os.path.join(d, "id"), 512, 768, 1024, 3, q)
    rank, bad, gbad, status, a_ok, tb = q[0]
    assert tb is None, tb
    assert bad == 0 and gbad == 0 and status == 0 and a_ok


def test_tp_k_split_padded_c(b2g, cuda, orc):
    """K-split with ldc > N (the reduce-scatter lands in scratch, then a strided copy)."""
    torch = cuda
    M, N, K, ldc = 256, 200, 300, 264
    uid = b2g.comm_unique_id()
    comm = b2g.comm_init(1, 0, uid)
    try:
        A = orc.uniform_f16((M, K), 5)
        B = orc.uniform_f16((K, N), 6)
        dA = torch.from_numpy(A.view(np.int16)).view(torch.float16).cuda()
        dB = torch.from_numpy(B.view(np.int16)).view(torch.float16).cuda()
        dC = torch.full((M, ldc), float("nan"), dtype=torch.float32, device="cuda")
        b2g.gemm_sharded_k(dA, dB, dC, M, N, K, comm, lda=K, ldb=N, ldc=ldc)
        torch.cuda.synchronize()
        assert b2g.device_status() == 0
        out = dC.cpu().numpy()
        assert_close(orc, out[:, :N], orc.gemm_f64(A, B), K)
        assert np.isnan(out[:, N:]).all()  # padding untouched
    finally:
        b2g.comm_destroy(comm)


@pytest.mark.parametrize("mode", ["k", "n"])
def test_tp_two_ranks(b2g, cuda, mode):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=shard_worker.nccl_tp_rank,
                             args=(mode, r, 2, os.path.join(d, "id"), 2048, 1536, 4096, 4, q))
                 for r in range(2)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    for rank, bad, gbad, status, a_ok, tb in res:
        assert tb is None, tb
        assert bad == 0 and gbad == 0 and status == 0 and a_ok, (rank, bad, gbad, status, a_ok)


def test_p2p_rs_single_rank(b2g, cuda):
    with tempfile.TemporaryDirectory() as d:
        q = _ListQueue()
        shard_worker.nccl_p2p_rs_rank(0, 1, os.path.join(d, "id"), 512, 768, 1024, 3, q)
    rank, bad, status, pad_ok, tb = q[0]
    assert tb is None, tb
    assert bad == 0 and status == 0 and pad_ok


@pytest.mark.parametrize("world,M,N,K", [(2, 2048, 1536, 4096), (2, 512, 1001, 777),
                                         (4, 4096, 2048, 4096), (8, 8192, 4096, 8192)])
def test_p2p_rs_multi_rank(b2g, cuda, world, M, N, K):
    """K-split GEMM with the reduce-scatter over peer memory: three calls in a row (slots
    reused under the epoch flags); N = 1001 stores through the generic kernel (rows not
    16-byte aligned) and reduces element by element."""
    if cuda.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=shard_worker.nccl_p2p_rs_rank,
                             args=(r, world, os.path.join(d, "id"), M, N, K, 3, q))
                 for r in range(world)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    for rank, bad, status, pad_ok, tb in res:
        assert tb is None, tb
        assert bad == 0 and status == 0 and pad_ok, (rank, bad, status, pad_ok)


@pytest.mark.parametrize("world,M,N,K,ldc", [(2, 2048, 1536, 4096, 1536), (2, 4096, 8192, 8192, 8200),
                                             (2, 520, 1000, 784, 1004), (4, 4096, 2048, 4096, 2048),
                                             (8, 8192, 4096, 8192, 4096)])
def test_p2p_rs_forms_give_the_same_bits(b2g, cuda, world, M, N, K, ldc):
    """Staged (copy-engine pushes), direct (remote stores) and fused (slot sum in the own
    slab's GEMM epilogue, one launch fewer) give the same C bits; 520 x 1000 x 784 has 260-row
    slabs (partial tiles) and 392-element K slabs (not a multiple of the 64-element stage);
    ldc > N leaves the pad alone."""
    if cuda.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=shard_worker.nccl_p2p_rs_forms_rank,
                             args=(r, world, os.path.join(d, "id"), M, N, K, ldc, q))
                 for r in range(world)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    for rank, same, launches, bad, status, tb in res:
        assert tb is None, tb
        assert same and bad == 0 and status == 0, (rank, same, bad, status)
        assert launches["fused"] == launches["direct"] - 1 == launches["staged"] - 1, launches


def test_chain_single_rank(b2g, cuda):
    with tempfile.TemporaryDirectory() as d:
        q = _ListQueue()
        shard_worker.nccl_chain_rank(0, 1, os.path.join(d, "id"), 512, 768, 1024, 3, 2, q)
    rank, rows, worst, status, b_ok, tb = q[0]
    assert tb is None, tb
    assert worst == 0 and status == 0 and b_ok


@pytest.mark.parametrize("world,M,N,K,panels", [(2, 2048, 1536, 4096, 6), (2, 640, 512, 200, 3),
                                                (4, 4096, 1024, 4096, 8), (8, 4096, 2048, 8192, 8)])
def test_chain_multi_rank(b2g, cuda, world, M, N, K, panels):
    """Copy-engine chain broadcast over `world` GPUs (skipped with fewer): three calls, the root
    rewriting B before each (the epoch flags and the 'done' handshake keep the panels of
    consecutive calls apart); every rank's slab rows checked and B bit-exact on every rank."""
    if cuda.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=shard_worker.nccl_chain_rank,
                             args=(r, world, os.path.join(d, "id"), M, N, K, panels, 3, q))
                 for r in range(world)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    for rank, rows, worst, status, b_ok, tb in res:
        assert tb is None, tb
        assert worst == 0 and status == 0 and b_ok, (rank, rows, worst, status, b_ok)
    assert sum(r[1] for r in res) == M


def test_n_chain_single_rank(b2g, cuda):
    with tempfile.TemporaryDirectory() as d:
        q = _ListQueue()
        shard_worker.nccl_n_chain_rank(0, 1, os.path.join(d, "id"), 512, 768, 1024, 3, 2, q)
    rank, nr, worst, status, a_ok, tb = q[0]
    assert tb is None, tb
    assert worst == 0 and status == 0 and a_ok


@pytest.mark.parametrize("world,M,N,K,panels", [(2, 2048, 1536, 2048, 6), (2, 300, 520, 200, 3)])
def test_n_chain_multi_rank(b2g, cuda, world, M, N, K, panels):
    """N-slab GEMM with A arriving through the copy-engine chain: three calls, the root
    rewriting A before each; every rank's column slab checked and A bit-exact on every rank."""
    if cuda.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=shard_worker.nccl_n_chain_rank,
                             args=(r, world, os.path.join(d, "id"), M, N, K, panels, 3, q))
                 for r in range(world)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    for rank, nr, worst, status, a_ok, tb in res:
        assert tb is None, tb
        assert worst == 0 and status == 0 and a_ok, (rank, nr, worst, status, a_ok)
    assert sum(r[1] for r in res) == N


def test_chain_broadcast_single_rank(b2g, cuda):
    with tempfile.TemporaryDirectory() as d:
        q = _ListQueue()
        shard_worker.nccl_chain_bcast_rank(0, 1, os.path.join(d, "id"), 512, 768, 1024, 3, 3, q)
    rank, rows, worst, status, b_ok, tb = q[0]
    assert tb is None, tb
    assert worst == 0 and status == 0 and b_ok


@pytest.mark.parametrize("world,M,N,K,panels,steps", [(2, 2048, 1536, 2048, 5, 4),
                                                      (2, 600, 520, 201, 3, 3),
                                                      (4, 4096, 1024, 4096, 8, 4),
                                                      (8, 8192, 2048, 4096, 8, 4)])
def test_chain_broadcast_multi_rank(b2g, cuda, world, M, N, K, panels, steps):
    """Double-buffered chain broadcast (bench.py's multi-GPU step): the broadcast of step i+1's
    B overlaps step i's slab GEMM; every step's rows checked, the B buffers bit-exact.
    K*N*2 = 209040 bytes in the second case is not a multiple of the 1 KiB panel unit."""
    if cuda.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=shard_worker.nccl_chain_bcast_rank,
                             args=(r, world, os.path.join(d, "id"), M, N, K, panels, steps, q))
                 for r in range(world)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    for rank, rows, worst, status, b_ok, tb in res:
        assert tb is None, tb
        assert worst == 0 and status == 0 and b_ok, (rank, rows, worst, status, b_ok)
    assert sum(r[1] for r in res) == M


@pytest.mark.parametrize("world,bad_rank", [(2, 1), (4, 2)])
def test_p2p_rs_peer_failure_reported_everywhere(b2g, cuda, world, bad_rank):
    """Peer-memory K-split: one rank passes ldc < N on the second of three calls.  That rank
    gets B2G_ERR_INVALID_ARG; the others' reductions see its status word, fill C with NaN and
    set the device error word to 7; the first and third calls are correct on every rank."""
    if cuda.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=shard_worker.nccl_p2p_rs_fail_rank,
                             args=(r, world, os.path.join(d, "id"), 512 * world, 768, 1024,
                                   bad_rank, q)) for r in range(world)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    for rank, outcomes, bad, status1, tb in res:
        assert tb is None, tb
        want = "invalid" if rank == bad_rank else "peer_failed"
        assert outcomes == ["ok", want, "ok"], (rank, outcomes, status1)
        assert bad == 0, (rank, bad)


def test_peer_leaves_between_steps_is_reported_within_the_limit(b2g, cuda):
    """Failure detection on 2 GPUs without a GPU fault: rank 1 stops taking part between steps.
    Rank 0's liveness check (b2g_comm_check, 3 s limit) returns B2G_ERR_TIMEOUT, with the
    communicator aborted, in a few seconds; its next chain call is refused (B2G_ERR_NCCL)
    without queueing work; teardown returns; the GPU still computes correctly."""
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=shard_worker.nccl_peer_leaves_rank,
                             args=(r, 2, os.path.join(d, "id"), q)) for r in range(2)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=120)
    for rank, first_ok, code, took, refused, ok_after, tb in res:
        assert tb is None, tb
        assert first_ok, rank
    r0 = res[0]
    assert r0[2] == b2g.ERR_TIMEOUT, r0
    assert r0[3] < 3.0 + 12.0, r0  # the limit plus the bounded drain of the aborted stream
    assert r0[4] == b2g.ERR_NCCL, r0
    assert r0[5], r0
