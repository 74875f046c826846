"""Host-side tests of the M-row-slab sharding (no GPU): the slab partition of the C library
and of shard.py agree and tile the rows exactly; the K-panel schedule; the broadcast/panel
pipeline on world_size-2 gloo ranks with an FP64 CPU stand-in for the per-panel GEMM; and a
rank that leaves before the collective makes the other rank's broadcast fail instead of
hanging.  The K-split (reduce-scatter) and N-slab (A broadcast, all-gather) schedules run the
same way on gloo ranks."""
import multiprocessing as mp
import os
import random
import socket
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import shard_worker  # noqa: E402


def _shard_mod():
    return shard_worker._load_pkg("shard")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_slab_partition_matches_library_and_tiles_rows(b2g):
    shard = _shard_mod()
    rng = random.Random(0)
    cases = [(32768, 8), (8192, 3), (7, 8), (0, 4), (1, 1), (129, 2)] + \
            [(rng.randrange(0, 5000), rng.randrange(1, 9)) for _ in range(40)]
    for M, world in cases:
        covered = []
        for r in range(world):
            lib = b2g.slab_rows(M, world, r)
            py = shard.slab_rows(M, world, r)
            assert lib == py
            covered.extend(range(py[0], py[0] + py[1]))
        assert covered == list(range(M))
        sizes = [shard.slab_rows(M, world, r)[1] for r in range(world)]
        assert max(sizes) - min(sizes) <= 1


def test_k_panels():
    shard = _shard_mod()
    assert shard.k_panels(8192, 4) == [(0, 2048), (2048, 4096), (4096, 6144), (6144, 8192)]
    assert shard.k_panels(100, 4) == [(0, 64), (64, 100)]
    assert shard.k_panels(0, 4) == [(0, 0)]
    for K in (1, 63, 64, 65, 1000, 32768):
        for P in (1, 2, 3, 8):
            b = shard.k_panels(K, P)
            assert b[0][0] == 0 and b[-1][1] == K
            assert all(x[1] == y[0] for x, y in zip(b, b[1:]))
            assert all(k0 % 64 == 0 for k0, _ in b)


@pytest.mark.parametrize("M,N,K,panels", [(96, 40, 192, 3), (7, 16, 64, 2), (130, 24, 100, 4)])
def test_gloo_two_rank_pipeline(M, N, K, panels):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=shard_worker.gloo_pipeline_rank,
                         args=(r, 2, port, M, N, K, panels, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    res.sort()
    for rank, rows, err, tb in res:
        assert tb is None, tb
        assert err < 1e-9, (rank, err)
    assert sum(r[1] for r in res) == M


def test_gloo_dead_rank_surfaces_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=shard_worker.gloo_dead_rank, args=(r, 2, port, q))
             for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (what, info)) for r, what, info in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1][0] == "left"
    assert res[0][0] == "error", res[0]


def _run_tp(mode, world, M, N, K, panels):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=shard_worker.gloo_tp_rank,
                         args=(mode, r, world, port, M, N, K, panels, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, err, gerr, tb in res:
        assert tb is None, tb
        assert 0 <= err < 1e-9 and 0 <= gerr < 1e-9, (rank, err, gerr)


@pytest.mark.parametrize("world,M,N,K", [(2, 96, 40, 192), (2, 8, 24, 1), (3, 30, 17, 100)])
def test_gloo_k_split_reduce_scatter(world, M, N, K):
    _run_tp("k", world, M, N, K, 1)


@pytest.mark.parametrize("world,M,N,K", [(2, 96, 40, 192), (2, 8, 24, 1), (3, 30, 17, 100)])
def test_gloo_k_split_peer_schedule(world, M, N, K):
    """The slab order, slot index and rank-order reduction of b2g_gemm_sharded_k_p2p."""
    _run_tp("kp", world, M, N, K, 1)


@pytest.mark.parametrize("world,M,N,K,panels", [(2, 200, 48, 64, 3), (2, 7, 5, 33, 2),
                                                (3, 130, 30, 20, 4)])
def test_gloo_n_slabs_all_gather(world, M, N, K, panels):
    _run_tp("n", world, M, N, K, panels)


@pytest.mark.parametrize("world,bad_rank", [(2, 1), (3, 0), (3, 2)])
def test_gloo_k_split_peer_failure_reported_everywhere(world, bad_rank):
    """One rank's invalid arguments on the second of three peer-memory K-split calls: that rank
    reports an invalid argument, every other rank a failed peer (C slab NaN), and the calls
    before and after are correct on every rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    M, N, K = 12 * world, 20, 70
    procs = [ctx.Process(target=shard_worker.gloo_p2p_fail_rank,
                         args=(r, world, port, M, N, K, bad_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, outcomes, err, tb in res:
        assert tb is None, tb
        want = "invalid" if rank == bad_rank else "peer_failed"
        assert outcomes == ["ok", want, "ok"], (rank, outcomes)
        assert 0 <= err < 1e-9, (rank, err)
