"""Rank bodies for the multi-process sharding tests (imported by spawned children)."""
import datetime
import os
import sys
import traceback

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _load_pkg(name):
    import importlib.util
    path = os.path.join(ROOT, "rdna4-gemm-wmma_b200", name + ".py")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _init_gloo(rank, world, port, timeout_s):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def gloo_pipeline_rank(rank, world, port, M, N, K, panels, out_q):
    """Run shard.sharded_gemm on CPU tensors with an FP64 numpy stand-in for the per-panel GEMM
    and report (rank, max error of the slab against the oracle)."""
    try:
        import torch
        from oracle import orc
        shard = _load_pkg("shard")
        dist = _init_gloo(rank, world, port, 60)
        row0, rows = shard.slab_rows(M, world, rank)
        A = orc.uniform_f16((M, K), 1)
        A_slab = torch.from_numpy(A[row0:row0 + rows].view(np.int16).copy()).view(torch.float16)
        if rank == 0:
            B = torch.from_numpy(orc.uniform_f16((K, N), 2).view(np.int16).copy()).view(torch.float16)
        else:
            B = torch.full((K, N), float("nan"), dtype=torch.float16)
        C_slab = torch.full((max(rows, 1), N), float("nan"), dtype=torch.float64)

        def cpu_gemm(A_view, B_view, C, r, n, k, beta, lda, ldb, ldc):
            prod = A_view[:r, :k].double() @ B_view[:k, :n].double()
            C[:r, :n] = prod if beta == 0.0 else C[:r, :n] + prod

        got = shard.sharded_gemm(A_slab, B, C_slab, M, N, K, panels=panels, gemm=cpu_gemm)
        assert got == (row0, rows)
        ref = orc.gemm_f64(A, orc.uniform_f16((K, N), 2), rows=(row0, row0 + rows))
        err = float(np.abs(C_slab[:rows].numpy() - ref).max()) if rows else 0.0
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, rows, err, None))
    except Exception:
        out_q.put((rank, -1, -1.0, traceback.format_exc()))


def gloo_dead_rank(rank, world, port, out_q):
    """Rank 1 leaves before the first collective; rank 0's broadcast must end with an error
    (the process-group timeout), not hang."""
    try:
        import torch
        shard = _load_pkg("shard")
        dist = _init_gloo(rank, world, port, 3)
        if rank == 1:
            out_q.put((rank, "left", None))
            out_q.close()
            out_q.join_thread()
            os._exit(0)
        B = torch.zeros((128, 64), dtype=torch.float16)
        A = torch.zeros((64, 128), dtype=torch.float16)
        C = torch.zeros((64, 64), dtype=torch.float64)
        try:
            shard.sharded_gemm(A, B, C, 128, 64, 128, panels=2,
                               gemm=lambda *a: None)
            out_q.put((rank, "no error", None))
        except Exception as e:  # the collective reports the missing peer
            out_q.put((rank, "error", type(e).__name__))
        out_q.close()
        out_q.join_thread()
        os._exit(0)
    except Exception:
        out_q.put((rank, "crash", traceback.format_exc()))


def nccl_sharded_rank(rank, world, uid_path, M, N, K, panels, out_q):
    """b2g_gemm_sharded on `world` GPUs (one process each); rank 0 publishes the NCCL id."""
    try:
        import time
        import torch
        from oracle import orc
        b2g = _load_pkg("b2g")
        torch.cuda.set_device(rank)
        if rank == 0:
            uid = b2g.comm_unique_id()
            with open(uid_path + ".tmp", "wb") as f:
                f.write(uid)
            os.replace(uid_path + ".tmp", uid_path)
        else:
            t0 = time.time()
            while not os.path.exists(uid_path):
                if time.time() - t0 > 60:
                    raise RuntimeError("no NCCL id from rank 0")
                time.sleep(0.05)
            uid = open(uid_path, "rb").read()
        comm = b2g.comm_init(world, rank, uid)
        row0, rows = b2g.slab_rows(M, world, rank)
        dA = torch.empty((max(rows, 1), K), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dA, rows * K, 1, row0 * K)
        dB = torch.full((K, N), float("nan"), dtype=torch.float16, device="cuda")
        if rank == 0:
            b2g.fill_uniform(dB, K * N, 2)
        dC = torch.full((max(rows, 1), N), float("nan"), dtype=torch.float32, device="cuda")
        b2g.gemm_sharded(dA, dB, dC, M, N, K, comm, root=0, k_panels=panels)
        torch.cuda.synchronize()
        status = b2g.device_status()
        # check a sample of this rank's rows against the oracle
        B = orc.uniform_f16((K, N), 2)
        sample = sorted(set([0, rows - 1] + list(range(0, rows, max(1, rows // 7))))) if rows else []
        worst = 0
        for r in sample:
            a = orc.uniform_f16((1, K), 1, (row0 + r) * K)
            ref = orc.gemm_f64(a, B)
            bad = orc.check(dC[r:r + 1].cpu().numpy(), ref, K, 1.0, 1.0)[0]
            worst = max(worst, bad)
        b_ok = bool(torch.equal(dB.cpu().view(torch.int16),
                                torch.from_numpy(B.view(np.int16))))
        b2g.comm_destroy(comm)
        out_q.put((rank, rows, worst, status, b_ok, None))
    except Exception:
        out_q.put((rank, -1, -1, -1, False, traceback.format_exc()))


def _f16(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x).view(np.int16).copy()).view(torch.float16)


def _cpu_gemm(A_view, B_view, C, r, n, k, beta, lda, ldb, ldc):
    """FP64 stand-in for the per-call GEMM of shard.py on CPU tensors."""
    prod = A_view[:r, :k].double() @ B_view[:k, :n].double()
    C[:r, :n] = prod if beta == 0.0 else C[:r, :n] + prod


def gloo_tp_rank(mode, rank, world, port, M, N, K, panels, out_q):
    """shard.sharded_gemm_k ("k"), its peer-memory schedule shard.sharded_gemm_k_p2p ("kp") or
    shard.sharded_gemm_n ("n") on CPU tensors with the FP64 stand-in; reports (rank, max error
    against the FP64 oracle of the rows/columns this rank owns, max error of the gathered C or
    0)."""
    try:
        import torch
        from oracle import orc
        shard = _load_pkg("shard")
        dist = _init_gloo(rank, world, port, 60)
        A = orc.uniform_f16((M, K), 1)
        B = orc.uniform_f16((K, N), 2)
        ref = orc.gemm_f64(A, B)
        gerr = 0.0
        if mode in ("k", "kp"):
            k0, kr = shard.slab_rows(K, world, rank)
            C_slab = torch.full((M // world, N), float("nan"), dtype=torch.float64)
            fn = shard.sharded_gemm_k if mode == "k" else shard.sharded_gemm_k_p2p
            row0, rows = fn(_f16(A[:, k0:k0 + kr]), _f16(B[k0:k0 + kr]), C_slab, M, N, K,
                            gemm=_cpu_gemm)
            err = float(np.abs(C_slab.numpy() - ref[row0:row0 + rows]).max()) if rows else 0.0
        else:
            n0, nr = shard.slab_rows(N, world, rank)
            A_t = _f16(A) if rank == 0 else torch.full((M, K), float("nan"), dtype=torch.float16)
            C_n = torch.full((M, max(nr, 1)), float("nan"), dtype=torch.float64)
            C_full = torch.full((M, N), float("nan"), dtype=torch.float64) if N % world == 0 else None
            got = shard.sharded_gemm_n(A_t, _f16(B[:, n0:n0 + nr]), C_n, M, N, K, panels=panels,
                                       C_full=C_full, gemm=_cpu_gemm)
            assert got == (n0, nr)
            err = float(np.abs(C_n[:, :nr].numpy() - ref[:, n0:n0 + nr]).max()) if nr else 0.0
            if C_full is not None:
                gerr = float(np.abs(C_full.numpy() - ref).max())
            assert np.array_equal(A_t.view(torch.int16).numpy(), A.view(np.int16))
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, err, gerr, None))
    except Exception:
        out_q.put((rank, -1.0, -1.0, traceback.format_exc()))


def _nccl_comm(b2g, rank, world, uid_path):
    import time
    if rank == 0:
        uid = b2g.comm_unique_id()
        with open(uid_path + ".tmp", "wb") as f:
            f.write(uid)
        os.replace(uid_path + ".tmp", uid_path)
    else:
        t0 = time.time()
        while not os.path.exists(uid_path):
            if time.time() - t0 > 60:
                raise RuntimeError("no NCCL id from rank 0")
            time.sleep(0.05)
        uid = open(uid_path, "rb").read()
    return b2g.comm_init(world, rank, uid)


def nccl_tp_rank(mode, rank, world, uid_path, M, N, K, panels, out_q):
    """b2g_gemm_sharded_k ("k") or b2g_gemm_sharded_n ("n") on `world` GPUs; reports
    (rank, failing elements of this rank's part on sampled rows, failing elements of the
    gathered C on sampled rows, device status, A-broadcast bit-exact)."""
    try:
        import torch
        from oracle import orc
        b2g = _load_pkg("b2g")
        torch.cuda.set_device(rank)
        comm = _nccl_comm(b2g, rank, world, uid_path)
        dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
        dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dA, M * K, 1)
        b2g.fill_uniform(dB, K * N, 2)
        B = orc.uniform_f16((K, N), 2)
        bad = gbad = 0
        a_ok = True
        if mode == "k":
            k0, kr = b2g.slab_rows(K, world, rank)
            rows = M // world
            dC = torch.full((rows, N), float("nan"), dtype=torch.float32, device="cuda")
            b2g.gemm_sharded_k(dA[:, k0:k0 + kr].contiguous(), dB[k0:k0 + kr].contiguous(), dC,
                               M, N, K, comm)
            torch.cuda.synchronize()
            for r in sorted(set([0, rows - 1, rows // 2, rows // 3])):
                a = orc.uniform_f16((1, K), 1, (rank * rows + r) * K)
                bad += orc.check(dC[r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K, 1.0, 1.0)[0]
        else:
            n0, nr = b2g.slab_rows(N, world, rank)
            if rank != 0:
                dA.fill_(float("nan"))
            dBn = dB[:, n0:n0 + nr].contiguous()
            dCn = torch.full((M, nr), float("nan"), dtype=torch.float32, device="cuda")
            dCf = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
            b2g.gemm_sharded_n(dA, dBn, dCn, M, N, K, comm, root=0, m_panels=panels, C_full=dCf)
            torch.cuda.synchronize()
            for r in sorted(set([0, M - 1, M // 2, M // 3, M // 7])):
                a = orc.uniform_f16((1, K), 1, r * K)
                ref = orc.gemm_f64(a, B)
                bad += orc.check(dCn[r:r + 1].cpu().numpy(), ref[:, n0:n0 + nr], K, 1.0, 1.0)[0]
                gbad += orc.check(dCf[r:r + 1].cpu().numpy(), ref, K, 1.0, 1.0)[0]
            a_ok = bool(torch.equal(dA.cpu().view(torch.int16),
                                    torch.from_numpy(orc.uniform_f16((M, K), 1).view(np.int16))))
        status = b2g.device_status()
        b2g.comm_destroy(comm)
        out_q.put((rank, bad, gbad, status, a_ok, None))
    except Exception:
        out_q.put((rank, -1, -1, -1, False, traceback.format_exc()))


def nccl_p2p_rs_rank(rank, world, uid_path, M, N, K, calls, out_q):
    """b2g_gemm_sharded_k_p2p on `world` GPUs: `calls` calls in a row with new operands each
    (another seed), the last one into a padded C (ldc > N); every call checked on sampled rows
    against the FP64 oracle, the padding left untouched."""
    try:
        import torch
        from oracle import orc
        b2g = _load_pkg("b2g")
        torch.cuda.set_device(rank)
        comm = _nccl_comm(b2g, rank, world, uid_path)
        plan = b2g.rs_plan_create(comm, M, N)
        k0, kr = b2g.slab_rows(K, world, rank)
        rows = M // world
        outs = []
        for c in range(calls):
            dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
            dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
            b2g.fill_uniform(dA, M * K, 1 + 10 * c)
            b2g.fill_uniform(dB, K * N, 2 + 10 * c)
            ldc = N + 8 if c == calls - 1 else N
            dC = torch.full((rows, ldc), float("nan"), dtype=torch.float32, device="cuda")
            b2g.gemm_sharded_k_p2p(plan, dA[:, k0:k0 + kr].contiguous(),
                                   dB[k0:k0 + kr].contiguous(), dC, M, N, K, lda=max(kr, 1),
                                   ldb=N, ldc=ldc)
            outs.append(dC)
        torch.cuda.synchronize()
        bad = 0
        pad_ok = True
        for c, dC in enumerate(outs):
            B = orc.uniform_f16((K, N), 2 + 10 * c)
            for r in sorted(set([0, rows - 1, rows // 2, rows // 3])):
                a = orc.uniform_f16((1, K), 1 + 10 * c, (rank * rows + r) * K)
                bad += orc.check(dC[r:r + 1, :N].cpu().numpy(), orc.gemm_f64(a, B), K, 1.0, 1.0)[0]
            if dC.shape[1] > N:
                pad_ok = pad_ok and bool(torch.isnan(dC[:, N:]).all())
        status = b2g.device_status()
        b2g.rs_plan_destroy(plan)
        b2g.comm_destroy(comm)
        out_q.put((rank, bad, status, pad_ok, None))
    except Exception:
        out_q.put((rank, -1, -1, False, traceback.format_exc()))


def nccl_p2p_rs_forms_rank(rank, world, uid_path, M, N, K, ldc, out_q):
    """b2g_gemm_sharded_k_p2p in its three forms on the same operands: staged (partials pushed
    by the copy engine; option rs_stage 1), direct (GEMMs store into the peers' slots; rs_stage
    0, rs_fused 0) and direct with the slots summed in the own slab's GEMM epilogue (rs_stage
    0, rs_fused 1).  C must be the same bits in all three and correct on sampled rows; the
    fused form launches one kernel fewer (no reduction kernel).  Reports (rank, C equal,
    {form: launches}, failing sampled elements, device status, traceback)."""
    try:
        import torch
        from oracle import orc
        b2g = _load_pkg("b2g")
        torch.cuda.set_device(rank)
        comm = _nccl_comm(b2g, rank, world, uid_path)
        plan = b2g.rs_plan_create(comm, M, N)  # rs_stage is on by default: staging buffers
        k0, kr = b2g.slab_rows(K, world, rank)
        rows = M // world
        dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
        dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dA, M * K, 31)
        b2g.fill_uniform(dB, K * N, 32)
        Ak, Bk = dA[:, k0:k0 + kr].contiguous(), dB[k0:k0 + kr].contiguous()
        forms = {"staged": (1, 0), "direct": (0, 0), "fused": (0, 1)}
        outs, launches = {}, {}
        old = {k: b2g.get_option(k) for k in ("rs_stage", "rs_fused")}
        try:
            for name, (stage, fused) in forms.items():
                b2g.set_option("rs_stage", stage)
                b2g.set_option("rs_fused", fused)
                dC = torch.full((rows, ldc), float("nan"), dtype=torch.float32, device="cuda")
                torch.cuda.synchronize()
                n0 = b2g.get_option("launches")
                b2g.gemm_sharded_k_p2p(plan, Ak, Bk, dC, M, N, K, lda=max(kr, 1), ldb=N, ldc=ldc)
                launches[name] = b2g.get_option("launches") - n0
                torch.cuda.synchronize()
                outs[name] = dC
        finally:
            for k, v in old.items():
                b2g.set_option(k, v)
        ref = outs["staged"]
        same = all(bool(torch.equal(o[:, :N].view(torch.int32), ref[:, :N].view(torch.int32)))
                   and bool(torch.isnan(o[:, N:]).all()) for o in outs.values())
        B = orc.uniform_f16((K, N), 32)
        bad = 0
        for r in sorted(set([0, rows - 1, rows // 2, rows // 3])):
            a = orc.uniform_f16((1, K), 31, (rank * rows + r) * K)
            bad += orc.check(ref[r:r + 1, :N].cpu().numpy(), orc.gemm_f64(a, B), K, 1.0, 1.0)[0]
        status = b2g.device_status()
        b2g.rs_plan_destroy(plan)
        b2g.comm_destroy(comm)
        out_q.put((rank, same, launches, bad, status, None))
    except Exception:
        out_q.put((rank, False, {}, -1, -1, traceback.format_exc()))


def nccl_chain_rank(rank, world, uid_path, M, N, K, panels, calls, out_q):
    """b2g_gemm_sharded_chain on `world` GPUs: `calls` calls in a row, the root writing a new B
    (another seed) before each; every call checked on sampled rows, and B bit-exact."""
    try:
        import torch
        from oracle import orc
        b2g = _load_pkg("b2g")
        torch.cuda.set_device(rank)
        comm = _nccl_comm(b2g, rank, world, uid_path)
        row0, rows = b2g.slab_rows(M, world, rank)
        dA = torch.empty((max(rows, 1), K), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dA, rows * K, 1, row0 * K)
        dB = torch.full((K, N), float("nan"), dtype=torch.float16, device="cuda")
        plan = b2g.chain_plan_create(comm, dB, K * N * 2, 0)
        stream = torch.cuda.current_stream()
        worst, b_ok = 0, True
        for c in range(calls):
            seed = 100 + c
            if rank == 0:
                b2g.fill_uniform(dB, K * N, seed, 0, stream.cuda_stream)
            dC = torch.full((max(rows, 1), N), float("nan"), dtype=torch.float32, device="cuda")
            b2g.gemm_sharded_chain(plan, dA, dC, M, N, K, k_panels=panels, stream=stream.cuda_stream)
            torch.cuda.synchronize()
            B = orc.uniform_f16((K, N), seed)
            for r in sorted(set([0, rows - 1, rows // 2])) if rows else []:
                a = orc.uniform_f16((1, K), 1, (row0 + r) * K)
                worst = max(worst, orc.check(dC[r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K, 1.0, 1.0)[0])
            b_ok = b_ok and bool(torch.equal(dB.cpu().view(torch.int16), torch.from_numpy(B.view(np.int16))))
        status = b2g.device_status()
        b2g.chain_plan_destroy(plan)
        b2g.comm_destroy(comm)
        out_q.put((rank, rows, worst, status, b_ok, None))
    except Exception:
        out_q.put((rank, -1, -1, -1, False, traceback.format_exc()))


def nccl_n_chain_rank(rank, world, uid_path, M, N, K, panels, calls, out_q):
    """b2g_gemm_sharded_n_chain on `world` GPUs: A (filled on the root only, a new seed before
    each call) reaches every rank through the copy-engine chain; this rank's column slab of C
    is checked on sampled rows, and A must be bit-exact on every rank."""
    try:
        import torch
        from oracle import orc
        b2g = _load_pkg("b2g")
        torch.cuda.set_device(rank)
        comm = _nccl_comm(b2g, rank, world, uid_path)
        n0, nr = b2g.slab_rows(N, world, rank)
        dA = torch.full((M, K), float("nan"), dtype=torch.float16, device="cuda")
        dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dB, K * N, 2)
        dBn = dB[:, n0:n0 + nr].contiguous()
        plan = b2g.chain_plan_create(comm, dA, M * K * 2, 0)
        stream = torch.cuda.current_stream()
        B = orc.uniform_f16((K, N), 2)
        worst, a_ok = 0, True
        for c in range(calls):
            seed = 200 + c
            if rank == 0:
                b2g.fill_uniform(dA, M * K, seed, 0, stream.cuda_stream)
            dCn = torch.full((M, max(nr, 1)), float("nan"), dtype=torch.float32, device="cuda")
            b2g.gemm_sharded_n_chain(plan, dBn, dCn, M, N, K, m_panels=panels, ldc=max(nr, 1),
                                     stream=stream.cuda_stream)
            torch.cuda.synchronize()
            for r in sorted(set([0, M - 1, M // 2, M // 3])):
                a = orc.uniform_f16((1, K), seed, r * K)
                ref = orc.gemm_f64(a, B)[:, n0:n0 + nr]
                worst = max(worst, orc.check(dCn[r:r + 1, :nr].cpu().numpy(), ref, K, 1.0, 1.0)[0])
            a_ok = a_ok and bool(torch.equal(dA.cpu().view(torch.int16),
                                             torch.from_numpy(orc.uniform_f16((M, K), seed).view(np.int16))))
        status = b2g.device_status()
        b2g.chain_plan_destroy(plan)
        b2g.comm_destroy(comm)
        out_q.put((rank, nr, worst, status, a_ok, None))
    except Exception:
        out_q.put((rank, -1, -1, -1, False, traceback.format_exc()))


def nccl_chain_bcast_rank(rank, world, uid_path, M, N, K, panels, steps, out_q):
    """Double-buffered broadcast along the copy-engine chain (b2g_chain_broadcast), the pattern
    of bench.py's multi-GPU line: two B buffers with a chain plan each; while step i's slab
    GEMM reads buffer i%2, the broadcast of step i+1's B (the root writes a new seed into it
    first) fills the other.  Every step's slab is checked on sampled rows against the FP64
    oracle with that step's B, and the last two B buffers must be bit-exact on every rank."""
    try:
        import torch
        from oracle import orc
        b2g = _load_pkg("b2g")
        torch.cuda.set_device(rank)
        comm = _nccl_comm(b2g, rank, world, uid_path)
        row0, rows = b2g.slab_rows(M, world, rank)
        dA = torch.empty((max(rows, 1), K), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dA, rows * K, 1, row0 * K)
        nbytes = K * N * 2
        dB = [torch.full((K, N), float("nan"), dtype=torch.float16, device="cuda")
              for _ in range(2)]
        plans = [b2g.chain_plan_create(comm, dB[b], nbytes, 0) for b in range(2)]
        s = torch.cuda.current_stream()
        sb = torch.cuda.Stream()
        bdone = [torch.cuda.Event() for _ in range(2)]
        gdone = [torch.cuda.Event() for _ in range(2)]

        def bcast(step):
            b = step % 2
            sb.wait_event(gdone[b])  # the GEMM that read this buffer two steps ago is done
            if rank == 0:
                b2g.fill_uniform(dB[b], K * N, 300 + step, 0, sb.cuda_stream)
            b2g.chain_broadcast(plans[b], nbytes, panels, stream=sb.cuda_stream)
            bdone[b].record(sb)

        torch.cuda.synchronize()
        bcast(0)
        outs = []
        for i in range(steps):
            if i + 1 < steps:
                bcast(i + 1)
            s.wait_event(bdone[i % 2])
            dC = torch.full((max(rows, 1), N), float("nan"), dtype=torch.float32, device="cuda")
            if rows:
                b2g.gemm(dA, dB[i % 2], dC, rows, N, K, stream=s.cuda_stream)
            gdone[i % 2].record(s)
            outs.append(dC)
        torch.cuda.synchronize()
        worst = 0
        for i, dC in enumerate(outs):
            B = orc.uniform_f16((K, N), 300 + i)
            for r in sorted(set([0, rows - 1, rows // 2])) if rows else []:
                a = orc.uniform_f16((1, K), 1, (row0 + r) * K)
                worst = max(worst, orc.check(dC[r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K,
                                             1.0, 1.0)[0])
        b_ok = True
        for i in range(max(0, steps - 2), steps):
            B = orc.uniform_f16((K, N), 300 + i)
            b_ok = b_ok and bool(torch.equal(dB[i % 2].cpu().view(torch.int16),
                                             torch.from_numpy(B.view(np.int16))))
        status = b2g.device_status()
        for p in plans:
            b2g.chain_plan_destroy(p)
        b2g.comm_destroy(comm)
        out_q.put((rank, rows, worst, status, b_ok, None))
    except Exception:
        out_q.put((rank, -1, -1, -1, False, traceback.format_exc()))


def gloo_p2p_fail_rank(rank, world, port, M, N, K, bad_rank, out_q):
    """shard.sharded_gemm_k_p2p with one rank's arguments invalid (a C slab narrower than N, the
    library's ldc < N) on the second of three calls: every rank must report the failure (the
    bad rank ValueError, the others PeerFailedError with a NaN C slab), and the calls before
    and after must be correct.  Reports (rank, [per-call outcome], max error of the good
    calls)."""
    try:
        import torch
        from oracle import orc
        shard = _load_pkg("shard")
        dist = _init_gloo(rank, world, port, 60)
        A = orc.uniform_f16((M, K), 1)
        B = orc.uniform_f16((K, N), 2)
        ref = orc.gemm_f64(A, B)
        k0, kr = shard.slab_rows(K, world, rank)
        rows = M // world
        outcomes, err = [], 0.0
        for call in range(3):
            width = N - 1 if (call == 1 and rank == bad_rank) else N
            C_slab = torch.full((rows, width), float("nan"), dtype=torch.float64)
            try:
                row0, _ = shard.sharded_gemm_k_p2p(_f16(A[:, k0:k0 + kr]), _f16(B[k0:k0 + kr]),
                                                   C_slab, M, N, K, gemm=_cpu_gemm)
                outcomes.append("ok")
                err = max(err, float(np.abs(C_slab.numpy() - ref[row0:row0 + rows]).max()))
            except shard.PeerFailedError:
                outcomes.append("peer_failed" if bool(torch.isnan(C_slab).all()) else "not_nan")
            except ValueError:
                outcomes.append("invalid")
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, outcomes, err, None))
    except Exception:
        out_q.put((rank, [], -1.0, traceback.format_exc()))


def nccl_p2p_rs_fail_rank(rank, world, uid_path, M, N, K, bad_rank, out_q):
    """b2g_gemm_sharded_k_p2p on `world` GPUs, three calls; on the second one rank passes an
    invalid ldc (< N).  That rank's call must return B2G_ERR_INVALID_ARG; every other rank's
    call is accepted, but its reduction finds the bad rank's status word and must leave NaN in
    C and the device error word at 7 (a peer's part failed).  The first and third calls must
    be correct on sampled rows.  Reports (rank, [per-call outcome], failing elements of the
    good calls, device status after the second call)."""
    try:
        import torch
        from oracle import orc
        b2g = _load_pkg("b2g")
        torch.cuda.set_device(rank)
        comm = _nccl_comm(b2g, rank, world, uid_path)
        plan = b2g.rs_plan_create(comm, M, N)
        k0, kr = b2g.slab_rows(K, world, rank)
        rows = M // world
        dA = torch.empty((M, K), dtype=torch.float16, device="cuda")
        dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dA, M * K, 1)
        b2g.fill_uniform(dB, K * N, 2)
        Ak, Bk = dA[:, k0:k0 + kr].contiguous(), dB[k0:k0 + kr].contiguous()
        B = orc.uniform_f16((K, N), 2)
        outcomes, bad, status1 = [], 0, None
        for call in range(3):
            dC = torch.full((rows, N), float("nan"), dtype=torch.float32, device="cuda")
            ldc = N - 1 if (call == 1 and rank == bad_rank) else N
            try:
                b2g.gemm_sharded_k_p2p(plan, Ak, Bk, dC, M, N, K, lda=max(kr, 1), ldb=N, ldc=ldc)
                rc = b2g.OK
            except b2g.B2GError as e:
                rc = e.code
            torch.cuda.synchronize()
            st = b2g.device_status()
            if call == 1:
                status1 = st
                if rc != b2g.OK:
                    outcomes.append("invalid" if rc == b2g.ERR_INVALID_ARG else "rc%d" % rc)
                else:
                    outcomes.append("peer_failed" if st == 7 and bool(torch.isnan(dC).all())
                                    else "status%d" % st)
            else:
                outcomes.append("ok" if rc == b2g.OK and st == 0 else "rc%d/status%d" % (rc, st))
                for r in sorted(set([0, rows - 1, rows // 2])):
                    a = orc.uniform_f16((1, K), 1, (rank * rows + r) * K)
                    bad += orc.check(dC[r:r + 1].cpu().numpy(), orc.gemm_f64(a, B), K, 1.0, 1.0)[0]
        b2g.rs_plan_destroy(plan)
        b2g.comm_destroy(comm)
        out_q.put((rank, outcomes, bad, status1, None))
    except Exception:
        out_q.put((rank, [], -1, -1, traceback.format_exc()))


def nccl_peer_leaves_rank(rank, world, uid_path, out_q):
    """Rank 1 leaves between steps: after one chain GEMM and one liveness check that every rank
    passes, it stops taking part (it stays alive, idle, until rank 0 is done, so no peer memory
    goes away under rank 0).  Rank 0's next liveness check must end within its limit with
    B2G_ERR_TIMEOUT (the communicator aborted, its all-reduce kernel returned); its next chain
    call must be refused without queueing work; plan and communicator teardown must return;
    and the GPU must still compute a correct GEMM.  NVLS is off (NCCL_NVLS_ENABLE=0).
    Reports (rank, first check ok, check code after the leave, seconds it took, code of the
    refused call, GEMM correct afterwards)."""
    import time
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import torch
        from oracle import orc
        b2g = _load_pkg("b2g")
        torch.cuda.set_device(rank)
        b2g.set_option("comm_timeout_ms", 20000)
        comm = _nccl_comm(b2g, rank, world, uid_path)
        M, N, K = 512 * world, 512, 1024
        row0, rows = b2g.slab_rows(M, world, rank)
        dA = torch.empty((rows, K), dtype=torch.float16, device="cuda")
        b2g.fill_uniform(dA, rows * K, 1, row0 * K)
        dB = torch.empty((K, N), dtype=torch.float16, device="cuda")
        if rank == 0:
            b2g.fill_uniform(dB, K * N, 2)
        plan = b2g.chain_plan_create(comm, dB, K * N * 2, 0)
        dC = torch.empty((rows, N), dtype=torch.float32, device="cuda")
        b2g.gemm_sharded_chain(plan, dA, dC, M, N, K, k_panels=2)
        torch.cuda.synchronize()
        b2g.comm_check(comm, 10000)
        first_ok = True
        done_flag = uid_path + ".rank0_done"
        if rank != 0:
            out_q.put((rank, first_ok, 0, 0.0, 0, True, None))
            out_q.close()
            out_q.join_thread()
            t0 = time.time()
            while not os.path.exists(done_flag) and time.time() - t0 < 120:
                time.sleep(0.05)
            os._exit(0)  # leaves without tearing anything down
        time.sleep(0.5)
        t0 = time.time()
        code = 0
        try:
            b2g.comm_check(comm, 3000)
        except b2g.B2GError as e:
            code = e.code
        took = time.time() - t0
        refused = 0
        try:
            b2g.gemm_sharded_chain(plan, dA, dC, M, N, K, k_panels=2)
        except b2g.B2GError as e:
            refused = e.code
        b2g.chain_plan_destroy(plan)
        b2g.comm_destroy(comm)
        # the GPU still works
        A = orc.uniform_f16((256, 512), 5)
        B = orc.uniform_f16((512, 384), 6)
        gA = torch.from_numpy(A.view(np.int16)).view(torch.float16).cuda()
        gB = torch.from_numpy(B.view(np.int16)).view(torch.float16).cuda()
        gC = torch.empty((256, 384), dtype=torch.float32, device="cuda")
        b2g.gemm(gA, gB, gC, 256, 384, 512)
        torch.cuda.synchronize()
        ok_after = orc.check(gC.cpu().numpy(), orc.gemm_f64(A, B), 512, 1.0, 1.0)[0] == 0
        with open(done_flag, "w") as f:
            f.write("done")
        out_q.put((rank, first_ok, code, took, refused, bool(ok_after), None))
    except Exception:
        try:
            with open(uid_path + ".rank0_done", "w") as f:
                f.write("failed")
        except OSError:
            pass
        out_q.put((rank, False, -1, -1.0, -1, False, traceback.format_exc()))
