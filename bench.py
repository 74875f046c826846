#!/usr/bin/env python
"""Benchmark of the B200 fp16 -> fp32 GEMM (BASELINE.json metric: TFLOP/s and % of B200
dense FP16 peak, 8192^3 fp16 -> fp32 GEMM, 1/2/4/8 GPU).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

One step = one 8192 x 8192 x 8192 GEMM per GPU.  With N > 1 (one
process per GPU under torchrun) rank r owns rows [8192 r, 8192 (r+1)) of an
(8192 N) x 8192 x 8192 GEMM: M-row slabs, C written locally with no reduction (weak
scaling: per-GPU work fixed), and every step also sends the whole B (128 MiB) from rank 0
to every rank along the library's copy-engine chain (b2g_chain_broadcast, peer copies over
NVLink, no SM).  B is double-buffered: step i+1's B travels while step i's slab GEMM runs.

Prints one JSON line (rank 0).  value = all ranks' FLOPs / max-over-ranks device time of K
steps with inputs resident in HBM.  e2e = the same metric through the public C ABI with
host buffers: each step copies A and B from pinned host memory and reads C back.
--impl reference times the reference's arithmetic on the host CPU (the oracle's blocked
port of GEMM_Naive, mmm.cpp:52-62; the HIP reference cannot run here).
"""
import argparse
import datetime
import json

import numpy as np
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SPEC_TFLOPS = 2250.0   # B200 dense fp16 tensor peak (spec)
M_PER_GPU = N_DIM = K_DIM = 8192
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}


def load_b2g():
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "b2g", os.path.join(ROOT, "rdna4-gemm-wmma_b200", "b2g.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.load()
    return mod


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def profiled_traffic(M, N, K, dtype="f16"):
    """DRAM bytes per launch of the top kernel from a committed ncu summary of this exact shape
    and operand type (`shape: M,N,K` and `traffic_bytes_per_launch:` lines), if any."""
    d = os.path.join(ROOT, "profiles")
    try:
        names = sorted(f for f in os.listdir(d) if f.endswith(".md"))
    except OSError:
        return None
    for f in names:
        shape = traffic = None
        dt = "f16"
        try:
            for line in open(os.path.join(d, f)):
                if line.startswith("shape:"):
                    shape = tuple(int(x) for x in line.split(":", 1)[1].strip().split(","))
                elif line.startswith("dtype:"):
                    dt = line.split(":", 1)[1].strip()
                elif line.startswith("traffic_bytes_per_launch:"):
                    traffic = float(line.split(":", 1)[1].strip())
        except (OSError, ValueError):
            continue
        if shape == (M, N, K) and dt == dtype and traffic is not None:
            return traffic
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, mx, pw = float(parts[1]), float(parts[2]), float(parts[3])
            except ValueError:
                continue
            if pw < 200:  # not under load (before the first / after the last launch)
                continue
            sms.append(sm)
            maxs.append(mx)
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxs),
                "reasons": sorted(reasons), "samples": len(sms)}


CPU_CHUNK_ROWS = 384  # rows of the 8192^3 problem per timed CPU chunk (both CPU legs)


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuGemm:
    """The oracle's blocked multithreaded port of GEMM_Naive (bit-exact) on the 8192^3 problem,
    timed in chunks of CPU_CHUNK_ROWS rows that cycle through the matrix.  Both CPU legs of the
    bench (the cpu_baseline key and --impl reference) use this one sample rule; the one-time
    widening of B to fp32 is charged pro rata to the rows computed."""

    def __init__(self, threads=None):
        from oracle import orc
        self.orc = orc
        self.A = orc.uniform_f16((M_PER_GPU, K_DIM), 1)
        self.B = orc.uniform_f16((K_DIM, N_DIM), 2)
        self.thr = threads or orc.nthreads()
        t0 = time.perf_counter()
        self.Bf = orc.widen_b(self.B, threads=self.thr)
        self.t_widen = time.perf_counter() - t0
        self.r0 = 0

    def chunk(self):
        """One chunk of rows; returns its charged seconds."""
        r0 = self.r0
        t0 = time.perf_counter()
        self.orc.gemm_f32_blocked(self.A, self.B, rows=(r0, r0 + CPU_CHUNK_ROWS), threads=self.thr,
                                  Bf=self.Bf)
        dt = time.perf_counter() - t0
        self.r0 = (r0 + CPU_CHUNK_ROWS) % (M_PER_GPU - CPU_CHUNK_ROWS + 1)
        return dt + self.t_widen * CPU_CHUNK_ROWS / M_PER_GPU

    @staticmethod
    def tflops(rows, secs):
        return 2.0 * rows * N_DIM * K_DIM / secs / 1e12


def cpu_baseline(seconds, threads=None):
    """The CPU baseline of the default line: chunks of the 8192^3 problem for about `seconds`
    (after one untimed chunk); returns TFLOP/s, rows done, seconds, threads."""
    g = CpuGemm(threads)
    g.chunk()
    rows, t = 0, 0.0
    while t < seconds or rows == 0:
        t += g.chunk()
        rows += CPU_CHUNK_ROWS
    return g.tflops(rows, t), rows, t, g.thr


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    g = CpuGemm()
    thr = g.thr
    # size each step (a whole number of chunks) so the whole run takes about a minute
    per_chunk = g.chunk()
    step_s = 60.0 / max(1, args.steps + args.warmup)
    chunks = max(1, int(round(step_s / per_chunk)))
    rows = chunks * CPU_CHUNK_ROWS
    for _ in range(args.warmup):
        for _ in range(chunks):
            g.chunk()
    times = []
    for _ in range(args.steps):
        times.append(sum(g.chunk() for _ in range(chunks)))
    tot = sum(times)
    val = g.tflops(rows * args.steps, tot)
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    line = {
        "impl": "reference",
        "metric": "gemm_tflops_8192cubed_fp16_fp32",
        "value": val,
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": tot / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 in, f32 accumulate/out",
        "data": "synthetic: seeded U[-1,1] fp16",
        "config": {"workload": "gemm 8192x8192x8192 row-major fp16->fp32 (BASELINE configs[1])",
                   "sample": "%d rows x 8192 x 8192 per step" % rows, "world_size": ws},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": thr, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": "%d rows per step (chunks of %d rows cycling through the "
                                   "8192) of the 8192^3 GEMM; blocked AVX2 port of GEMM_Naive "
                                   "(mmm.cpp:52-62), bit-exact; B widening charged pro rata"
                                   % (rows, CPU_CHUNK_ROWS)},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is HIP/rocBLAS for AMD gfx12 and cannot run on this box; this "
                "arm is the CPU port of its arithmetic",
    }
    print(json.dumps(line), flush=True)
    return 0


ALL_CONFIGS = [
    ("configs[0]", ["--shape", "1024,1024,1024"]),
    ("configs[1]", ["--shape", "8192,8192,8192"]),
    ("configs[2]", ["--workload", "contraction5d"]),
    ("configs[3]", ["--shape", "16384,16384,4096"]),
    ("configs[3]", ["--shape", "8192,28672,8192"]),
    ("configs[3]", ["--shape", "128,8192,8192"]),
    ("configs[4] on one GPU", ["--shape", "32768,32768,32768"]),
]


def run_all_configs(args):
    """One kernel-loop line per BASELINE config on one GPU, each from its own process (so every
    config starts from a fresh memory pool), with clocks and cuBLAS side by side.  32768^3 runs
    at most 20 steps (61 ms each)."""
    rc = 0
    for label, extra in ALL_CONFIGS:
        steps = args.steps if "32768" not in extra[-1] else min(args.steps, 20)
        cmd = [sys.executable, os.path.abspath(__file__)] + extra + [
            "--steps", str(steps), "--warmup", str(args.warmup)] + (["--no-graph"] if args.no_graph else [])
        res = subprocess.run(cmd, capture_output=True, text=True)
        lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
        if res.returncode != 0 or not lines:
            rc = res.returncode or 1
            print(json.dumps({"baseline_config": label, "args": extra, "rc": res.returncode,
                              "stderr_tail": res.stderr[-400:]}), flush=True)
            continue
        line = json.loads(lines[-1])
        line["baseline_config"] = label
        print(json.dumps(line), flush=True)
    return rc


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b2g", choices=["b2g", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=40)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--workload", default="gemm8192",
                    choices=["gemm8192", "sharded32768", "contraction5d", "tp_k"],
                    help="gemm8192: BASELINE configs[1] per GPU (the default line); "
                         "contraction5d: BASELINE configs[2] through the contraction entry point "
                         "(C[a,b,i,n] = sum A[a,b,i,j,k] B[j,k,n], a8 b16 i64 j64 k128 n4096); "
                         "sharded32768: BASELINE configs[4], one 32768^3 GEMM as M-row slabs "
                         "over the N GPUs, B broadcast in K panels inside every step; "
                         "tp_k: tensor-parallel K-split GEMM (8192^3 or --shape) whose partials "
                         "are reduce-scattered over the N GPUs inside every step")
    ap.add_argument("--bcast", default="chain", choices=["chain", "nccl"],
                    help="sharded32768: how B reaches the ranks each step (copy-engine chain, "
                         "or ncclBroadcast)")
    ap.add_argument("--tp", default="p2p", choices=["p2p", "nccl"],
                    help="tp_k: reduce-scatter fused into the GEMMs over peer memory, or "
                         "ncclReduceScatter after the GEMM")
    ap.add_argument("--rs-form", default="staged", choices=["staged", "direct", "fused"],
                    help="tp_k --tp p2p: staged = peers' partials computed locally and pushed "
                         "by the copy engine during the next GEMM; direct = the GEMMs store into "
                         "the peers' slots; fused = direct, with the slots summed in the own "
                         "slab's GEMM epilogue (all three give the same bits)")
    ap.add_argument("--shape", default=None,
                    help="M,N,K: time this row-major GEMM instead of 8192^3 (device-resident "
                         "kernel loop only; used for the other BASELINE shapes and for profiling)")
    ap.add_argument("--dtype", default="f16", choices=["f16", "bf16", "e4m3", "e5m2"],
                    help="operand type (f16 = BASELINE's; the others are secondary lines)")
    ap.add_argument("--out", default="f32", choices=["f32", "f16", "bf16"],
                    help="type C is stored in (the fused epilogue; f32 = BASELINE's). Kernel loop only")
    ap.add_argument("--bias", action="store_true",
                    help="add a per-column fp32 bias in the epilogue. Kernel loop only")
    ap.add_argument("--kernel-only", action="store_true",
                    help="device-resident GEMM steps only (no e2e, CPU baseline or clock "
                         "sampling): the command profiled with ncu")
    ap.add_argument("--graph", action="store_true",
                    help="one GPU: also time the step replayed from a CUDA graph (device time "
                         "per step without host launch gaps), this library's and cuBLAS's in "
                         "turn (on by default for one GPU; kept for older command lines)")
    ap.add_argument("--no-graph", action="store_true", help="skip the CUDA graph timing")
    ap.add_argument("--option", action="append", default=[], metavar="KEY=VALUE",
                    help="set a library option (b2g_set_option) before timing; repeatable")
    ap.add_argument("--all-configs", action="store_true",
                    help="one JSON line per BASELINE config on one GPU (1024^3, 8192^3, the "
                         "configs[2] contraction, the three configs[3] shapes, 32768^3), each "
                         "with clocks and cuBLAS side by side")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.all_configs:
        return run_all_configs(args)
    args.sample_clocks = not args.kernel_only

    import torch
    import torch.distributed as dist

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    b2g = load_b2g()
    for opt in args.option:
        key, _, val = opt.partition("=")
        b2g.set_option(key, int(val))
    if args.workload == "sharded32768":
        return run_sharded(args, torch, dist, b2g, ws, rank, local, dev)
    if args.workload == "tp_k":
        return run_tp_k(args, torch, dist, b2g, ws, rank, local, dev)

    M, N, K = M_PER_GPU, N_DIM, K_DIM
    contraction = args.workload == "contraction5d"
    if contraction:
        # the contraction's GEMM view is M = a*b*i, K = j*k, N = n
        c5 = dict(a=8, b=16, i=64, j=64, k=128, n=4096)
        M, N, K = c5["a"] * c5["b"] * c5["i"], c5["n"], c5["j"] * c5["k"]
        a_shape = (c5["a"], c5["b"], c5["i"], c5["j"], c5["k"])
        b_shape = (c5["j"], c5["k"], c5["n"])
        c_shape = (c5["a"], c5["b"], c5["i"], c5["n"])
        rowmajor = lambda sh: tuple(int(np.prod(sh[d + 1:])) for d in range(len(sh)))
        args.kernel_only = True
    if args.shape:
        # another BASELINE shape (configs[0], [2] as its GEMM view, [3]); kernel loop only
        M, N, K = (int(x) for x in args.shape.split(","))
        args.kernel_only = True
    flops = 2.0 * M * N * K
    stream = torch.cuda.current_stream()
    dt = {"f16": 0, "bf16": 1, "e4m3": 2, "e5m2": 3}[args.dtype]
    tdt = {0: torch.float16, 1: torch.bfloat16, 2: torch.uint8, 3: torch.uint8}[dt]
    epilogue = args.out != "f32" or args.bias
    if dt or epilogue:
        args.kernel_only = True  # secondary types and epilogues: device-resident kernel loop only
    dA = torch.empty((M, K), dtype=tdt, device=dev)
    dB = torch.empty((K, N), dtype=tdt, device=dev)
    c_dt = {"f32": 4, "f16": 0, "bf16": 1}[args.out]
    dC = torch.empty((M, N), device=dev,
                     dtype={"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[args.out])
    dBias = torch.randn(N, device=dev) if args.bias else None
    # rank r's slab of the (M*ws) x K matrix A; B generated on rank 0
    b2g.fill_uniform(dA, M * K, 1, rank * M * K, stream, dtype=dt)
    if rank == 0:
        b2g.fill_uniform(dB, K * N, 2, 0, stream, dtype=dt)
    torch.cuda.synchronize()
    # N > 1: B travels from rank 0 along the copy-engine chain (peer copies over NVLink, no SM)
    # inside every step.  Two B buffers with a chain plan each: while step i's slab GEMM reads
    # buffer i % 2, the broadcast of step i+1's B fills the other one, so every timed step
    # moves the whole B to every rank and computes one slab GEMM.
    chain = None
    if ws > 1 and (contraction or dt or epilogue):
        dist.broadcast(dB, src=0)  # secondary lines: B replicated once at set-up
        torch.cuda.synchronize()
    elif ws > 1:
        comm = library_comm(torch, dist, b2g, ws, rank, dev)
        dB2 = torch.empty_like(dB)
        if rank == 0:
            dB2.copy_(dB)
        bufs = [dB, dB2]
        plans = [b2g.chain_plan_create(comm, b, K * N * dB.element_size(), 0) for b in bufs]
        sb = torch.cuda.Stream(dev)
        chain = {"comm": comm, "bufs": bufs, "plans": plans, "sb": sb, "n": 0,
                 "bdone": [torch.cuda.Event() for _ in range(2)],
                 "gdone": [torch.cuda.Event() for _ in range(2)],
                 "bytes": K * N * dB.element_size(), "panels": 8}

        def bcast(i):
            b = i % 2
            chain["sb"].wait_event(chain["gdone"][b])  # the GEMM that read this buffer is done
            b2g.chain_broadcast(chain["plans"][b], chain["bytes"], chain["panels"],
                                stream=chain["sb"].cuda_stream)
            chain["bdone"][b].record(chain["sb"])

        bcast(0)  # step 0's B; every step then broadcasts the next step's
        torch.cuda.synchronize()
        sys.stderr.write("rank %d/%d: B (%d MiB) along a copy-engine chain of %d ranks every "
                         "step\n" % (rank, ws, chain["bytes"] >> 20, ws))

    def step(st=None):
        st = stream if st is None else st
        if chain is not None:
            i = chain["n"]
            b = i % 2
            bcast(i + 1)
            st.wait_event(chain["bdone"][b])
            b2g.gemm(dA, chain["bufs"][b], dC, M, N, K, K, N, N, st)
            chain["gdone"][b].record(st)
            chain["n"] = i + 1
        elif contraction:
            b2g.contract5d(dA, a_shape, rowmajor(a_shape), dB, b_shape, rowmajor(b_shape), dC,
                           c_shape, rowmajor(c_shape), st)
        elif epilogue:
            b2g.gemm_epilogue(dA, dB, dC, M, N, K, dtype=dt, bias=dBias, c_dtype=c_dt,
                              stream=st)
        elif dt:
            b2g.gemm_typed(dA, dB, dC, M, N, K, dt, stream=st)
        else:
            b2g.gemm(dA, dB, dC, M, N, K, K, N, N, st)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if b2g.device_status() != 0:
        raise SystemExit("device-side wait timed out during warm-up")

    # The timed region (value): K back-to-back steps with events only around the whole loop, so
    # consecutive launches overlap as they do for a user (programmatic dependent launch).
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local) if args.sample_clocks else None
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    launches0 = b2g.get_option("launches")
    t_start.record(stream)
    if chain is not None:
        chain["sb"].wait_stream(stream)  # the timed broadcasts start inside the region
    for i in range(args.steps):
        step()
    if chain is not None:
        stream.wait_stream(chain["sb"])  # ... and the last one ends inside it
    t_end.record(stream)
    launches = b2g.get_option("launches") - launches0
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    if ws > 1:
        dist.barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    # Kernel duration for the roofline: a second pass with an event pair around every launch
    # (the events keep launches from overlapping, so this is each launch on its own).
    n_ev = min(args.steps, 200)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(n_ev)]
    for i in range(n_ev):
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    path = b2g.PATH_NAMES.get(b2g.last_path(), "?")
    if b2g.device_status() != 0:
        raise SystemExit("device-side wait timed out during the timed region")
    chain_info = None
    if chain is not None:
        # spot check on every rank: row 0 of the last step's slab against the FP64 product
        # with the B this rank received, and that B identical on every rank (checksums)
        last = chain["bufs"][(chain["n"] - 1) % 2]
        bad = row_out_of_tolerance(torch, dC[:1], dA[:1], last, K)
        sums = []
        for b in chain["bufs"]:
            cs = b.view(torch.int16).to(torch.int64).sum().reshape(1)
            lo, hi = cs.clone(), cs.clone()
            dist.all_reduce(lo, op=dist.ReduceOp.MIN)
            dist.all_reduce(hi, op=dist.ReduceOp.MAX)
            sums.append(bool(lo.item() == hi.item()))
        chk = torch.tensor([bad], dtype=torch.int64, device=dev)
        dist.all_reduce(chk, op=dist.ReduceOp.MAX)
        for p in chain["plans"]:
            b2g.chain_plan_destroy(p)
        b2g.comm_destroy(chain["comm"])
        chain_info = {"ranks_in_chain": ws, "bytes_per_step": chain["bytes"],
                      "panels": chain["panels"], "row0_out_of_tolerance_max_over_ranks":
                      int(chk.item()), "b_identical_on_all_ranks": all(sums)}
    if ws > 1:
        dist.barrier()

    value = flops * ws * args.steps / (elapsed_ms * 1e-3) / 1e12
    avg_launch_ms = statistics.mean(launch_ms)
    achieved = flops / (avg_launch_ms * 1e-3) / 1e12

    # ---- device time per step from CUDA graph replay (no host launch gaps), ours and cuBLAS's,
    # their replays interleaved so that both see the same clocks under the power cap
    graph = None
    if not args.no_graph and ws == 1:
        calls = max(1, min(args.steps, 20 if flops < 2 ** 37 else 5))
        fns = [lambda: step(torch.cuda.current_stream())]
        if dt == 0 and not epilogue and not args.no_cublas:
            fns.append(lambda: torch.mm(dA, dB, out_dtype=torch.float32))
        us = graph_us_per_call(torch, fns, calls)
        graph = {"us_per_step": us[0], "value": flops / (us[0] * 1e-6) / 1e12, "unit": "TFLOP/s",
                 "calls_per_graph": calls, "replays": 10, "interleaved": len(us) > 1}
        if len(us) > 1:
            graph["cublas_us_per_step"] = us[1]
            graph["cublas_value"] = flops / (us[1] * 1e-6) / 1e12

    # ---- end to end through the C ABI with host buffers (pipelined over 3 streams)
    e2e = None
    cublas = None
    if not args.kernel_only:
        e2e = e2e_run(torch, b2g, dev, M, N, K, rank, ws, args.e2e_steps, dist if ws > 1 else None)
    if (rank == 0 and ws == 1 and not args.no_cublas and dt == 0 and not epilogue and
            (args.shape or contraction or not args.kernel_only)):
        cublas = cublas_side_by_side(torch, dA, dB, dC, local, min(args.steps, 1000))

    peaks, peaks_src = measured_peaks()
    # a loop of back-to-back launches longer than ~0.25 s runs under the power cap: compare with
    # the sustained (power-capped) library figure, otherwise with the burst one
    sustained = elapsed_ms > 250.0
    peak = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
    peak_note = ""
    if dt >= 2:  # fp8 tensor rate is twice fp16/bf16 (nominal 4.5 vs 2.25 PFLOP/s dense)
        peak *= 2.0
        peak_note = " x2 (fp8 = 2x the measured 16-bit rate)"
    # Roofline of the kernel: tensor-bound unless the shape's arithmetic intensity is below the
    # ridge of the measured peaks (then HBM-bound, achieved = algorithmic bytes / launch time).
    esz = 2 if dt < 2 else 1
    c_esz = 4 if args.out == "f32" else 2
    alg_bytes = float(esz * M * K + esz * K * N + c_esz * M * N + (4 * N if args.bias else 0))
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    ridge = peak * 1e12 / (hbm * 1e9)
    if flops / alg_bytes < ridge:
        roofline = {"bound": "hbm", "achieved": alg_bytes / (avg_launch_ms * 1e-3) / 1e9,
                    "peak": hbm, "unit": "GB/s",
                    "frac": alg_bytes / (avg_launch_ms * 1e-3) / 1e9 / hbm,
                    "traffic": None if epilogue else profiled_traffic(M, N, K, args.dtype),
                    "peak_source": "%s hbm_gbs" % peaks_src,
                    "bytes_per_launch": alg_bytes, "flops_per_launch": flops,
                    "avg_launch_ms": avg_launch_ms, "tensor_tflops": achieved}
    else:
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak,
                    "traffic": None if epilogue else profiled_traffic(M, N, K, args.dtype),
                    "peak_source": "%s %s%s" % (peaks_src, "bf16_tflops_sustained" if sustained
                                                else "bf16_tflops", peak_note),
                    "flops_per_launch": flops, "bytes_per_launch": alg_bytes,
                    "avg_launch_ms": avg_launch_ms}
    roofline["kernel"] = "gemm_tc_kernel"
    # per-launch spread of the same pass: the minimum is what the reference reports
    # (getBestTiming, mmm.cpp:1376)
    roofline["min_launch_ms"] = min(launch_ms)
    roofline["median_launch_ms"] = statistics.median(launch_ms)
    roofline["launches_timed"] = len(launch_ms)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline and not args.kernel_only:
        v, rows, secs, thr = cpu_baseline(args.cpu_seconds)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": thr, "kind": "port",
               "cpu_model": cpu_model(),
               "sample": "%d rows of the 8192^3 GEMM in chunks of %d rows (%.1f s); blocked "
                         "AVX2 port of GEMM_Naive (mmm.cpp:52-62), bit-exact; B widening charged "
                         "pro rata" % (rows, CPU_CHUNK_ROWS, secs)}
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    metric = "gemm_tflops_8192cubed_fp16_fp32"
    if contraction:
        metric = "contraction_tflops_a8b16i64j64k128n4096_fp16_fp32"
    if args.shape:
        metric = "gemm_tflops_%dx%dx%d_fp16_fp32" % (M, N, K)
    if dt:
        metric = metric.replace("fp16", args.dtype)
    if args.out != "f32":
        metric = metric.replace("_fp32", "_" + args.out + "out")
    if args.bias:
        metric += "_bias"
    line = {
        "metric": metric,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "%s in, f32 accumulate, %s out%s" % (args.dtype, args.out,
                                                       " + f32 column bias" if args.bias else ""),
        "data": "synthetic: seeded U[-1,1] %s generated on the device (b2g_fill_uniform)" % args.dtype,
        "config": {
            "workload": ("contraction C[a,b,i,n] = sum_{j,k} A[a,b,i,j,k] B[j,k,n], a8 b16 i64 j64 "
                         "k128 n4096, contiguous operands through b2g_contract5d (BASELINE "
                         "configs[2]; GEMM view %dx%dx%d)" % (M, N, K)) if contraction
                        else ("gemm %dx%dx%d row-major fp16->fp32 (kernel loop)" % (M, N, K)) if args.shape
                        else "gemm 8192x8192x8192 row-major fp16->fp32 per GPU (BASELINE configs[1]);"
                             " N>1: M-row slabs of a (8192N)x8192x8192 GEMM, B (128 MiB) sent from "
                             "rank 0 along the copy-engine chain every step, double-buffered (step "
                             "i+1's B travels while step i's slab GEMM runs)",
            "M": M, "N": N, "K": K, "world_size": ws, "path": path,
            "broadcast": chain_info,
            "l2": "inputs+output %.0f MiB per GPU (%s 126 MB L2)" % (
                alg_bytes / 2**20, "> : no flush needed" if alg_bytes > 126e6 else
                "< : steps may hit L2"),
            "frac_of_spec_2250": value / ws / SPEC_TFLOPS,
        },
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "cublas_side_by_side": cublas,
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if graph is not None:
        line["graph"] = graph
    if args.option:
        line["config"]["options"] = dict(o.partition("=")[::2] for o in args.option)
    if clocks and clocks.get("sm_mhz"):
        # clock-normalised rate: the per-GPU value per GHz of the median SM clock under load
        clocks["tflops_per_ghz_per_gpu"] = value / ws / (clocks["sm_mhz"] / 1000.0)
    if cublas and cublas.get("value") and (cublas.get("clocks") or {}).get("sm_mhz"):
        cublas["clocks"]["tflops_per_ghz"] = cublas["value"] / (cublas["clocks"]["sm_mhz"] / 1000.0)
    print(json.dumps(line), flush=True)
    return 0


def run_sharded(args, torch, dist, b2g, ws, rank, local, dev):
    """C[32768,32768] = A.B with A/C as M-row slabs over the ws ranks and
    B broadcast from rank 0 in K panels inside every step (b2g_gemm_sharded over the
    library's own NCCL communicator).  Strong scaling: the total work is fixed."""
    import numpy as np
    M = N = K = 32768
    uid = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        uid.copy_(torch.from_numpy(np.frombuffer(b2g.comm_unique_id(), dtype=np.uint8).copy()))
    if ws > 1:
        dist.broadcast(uid, src=0)
    comm = b2g.comm_init(ws, rank, bytes(uid.cpu().numpy().tobytes()))
    row0, rows = b2g.slab_rows(M, ws, rank)
    stream = torch.cuda.current_stream()
    dA = torch.empty((rows, K), dtype=torch.float16, device=dev)
    dB = torch.empty((K, N), dtype=torch.float16, device=dev)
    dC = torch.empty((rows, N), dtype=torch.float32, device=dev)
    b2g.fill_uniform(dA, rows * K, 1, row0 * K, stream)
    if rank == 0:
        b2g.fill_uniform(dB, K * N, 2, 0, stream)
    panels = 8
    plan = None
    if args.bcast == "chain":
        plan = b2g.chain_plan_create(comm, dB, K * N * 2, 0)

    def step():
        if plan is not None:
            b2g.gemm_sharded_chain(plan, dA, dC, M, N, K, k_panels=panels, stream=stream)
        else:
            b2g.gemm_sharded(dA, dB, dC, M, N, K, comm, root=0, k_panels=panels, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    launches0 = b2g.get_option("launches")
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    launches = b2g.get_option("launches") - launches0
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # spot check: first row of every rank's slab (B on each rank arrived through the broadcast)
    bad = row_out_of_tolerance(torch, dC[:1], dA[:1], dB, K)
    status = b2g.device_status()
    if ws > 1:
        chk = torch.tensor([bad, abs(status)], dtype=torch.int64, device=dev)
        dist.all_reduce(chk, op=dist.ReduceOp.MAX)
        bad, status = int(chk[0].item()), int(chk[1].item())
    if ws > 1:
        dist.barrier()
    if plan is not None:
        b2g.chain_plan_destroy(plan)
    b2g.comm_destroy(comm)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        flops = 2.0 * M * N * K
        print(json.dumps({
            "metric": "sharded_gemm_tflops_32768cubed_fp16_fp32", "value": flops * args.steps / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 in, f32 accumulate/out",
            "data": "synthetic: seeded U[-1,1] fp16 generated on the device",
            "config": {"workload": "gemm 32768^3 as M-row slabs over N GPUs, B broadcast from rank 0 "
                                   "in %d K panels every step (BASELINE configs[4])" % panels,
                       "rows_per_rank": rows, "k_panels": panels,
                       "broadcast": ("copy-engine chain (peer copies + stream memory ops, no SM)"
                                     if plan is not None else "NCCL broadcast")},
            "row0_out_of_tolerance": bad, "device_status": status,
            "gpu_launches": launches}), flush=True)
    return 0


def library_comm(torch, dist, b2g, ws, rank, dev):
    """The library's own NCCL communicator over the ws ranks (id broadcast from rank 0)."""
    import numpy as np
    uid = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        uid.copy_(torch.from_numpy(np.frombuffer(b2g.comm_unique_id(), dtype=np.uint8).copy()))
    if ws > 1:
        dist.broadcast(uid, src=0)
    return b2g.comm_init(ws, rank, bytes(uid.cpu().numpy().tobytes()))


def run_tp_k(args, torch, dist, b2g, ws, rank, local, dev):
    """Tensor-parallel K-split GEMM: rank r holds the K slab of A and B, and every step ends
    with rows [r*M/ws, (r+1)*M/ws) of C = sum over ranks of A_r.B_r on rank r (the partials
    reduce-scattered over peer memory inside the GEMMs, or by ncclReduceScatter).  Strong
    scaling: the total work is fixed."""
    M, N, K = (int(x) for x in args.shape.split(",")) if args.shape else (8192, 8192, 8192)
    comm = library_comm(torch, dist, b2g, ws, rank, dev)
    k0, kr = b2g.slab_rows(K, ws, rank)
    rows = M // ws
    stream = torch.cuda.current_stream()
    # the full seeded A and B on every rank (for the spot check); each rank multiplies its slab
    A = torch.empty((M, K), dtype=torch.float16, device=dev)
    B = torch.empty((K, N), dtype=torch.float16, device=dev)
    b2g.fill_uniform(A, M * K, 1, 0, stream)
    b2g.fill_uniform(B, K * N, 2, 0, stream)
    dA = A[:, k0:k0 + kr].contiguous()
    dB = B[k0:k0 + kr].contiguous()
    dC = torch.empty((rows, N), dtype=torch.float32, device=dev)
    b2g.set_option("rs_stage", 1 if args.rs_form == "staged" else 0)
    b2g.set_option("rs_fused", 1 if args.rs_form == "fused" else 0)
    plan = b2g.rs_plan_create(comm, M, N) if args.tp == "p2p" else None

    def step():
        if plan is not None:
            b2g.gemm_sharded_k_p2p(plan, dA, dB, dC, M, N, K, stream=stream)
        else:
            b2g.gemm_sharded_k(dA, dB, dC, M, N, K, comm, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    launches0 = b2g.get_option("launches")
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    launches = b2g.get_option("launches") - launches0
    torch.cuda.synchronize()
    t = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # spot check: first row of every rank's part against the FP64 product of the full operands
    bad = row_out_of_tolerance(torch, dC[:1], A[rank * rows:rank * rows + 1], B, K)
    status = b2g.device_status()
    if ws > 1:
        chk = torch.tensor([bad, abs(status)], dtype=torch.int64, device=dev)
        dist.all_reduce(chk, op=dist.ReduceOp.MAX)
        bad, status = int(chk[0].item()), int(chk[1].item())
        dist.barrier()
    if plan is not None:
        b2g.rs_plan_destroy(plan)
    b2g.comm_destroy(comm)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        flops = 2.0 * M * N * K
        value = flops * args.steps / (ms * 1e-3) / 1e12
        peaks, src = measured_peaks()
        # fused compute + collective: the target time per step is the slower of the per-rank
        # GEMM at the measured sustained peak and the partials this rank sends over NVLink at
        # the measured 770 GB/s peer bandwidth
        link = 770.0
        t_gemm = flops / ws / (peaks["bf16_tflops_sustained"] * 1e12)
        nv_bytes = (ws - 1) / ws * M * N * 4.0
        t_link = nv_bytes / (link * 1e9)
        target = max(t_gemm, t_link)
        print(json.dumps({
            "metric": "tp_ksplit_gemm_tflops_%dx%dx%d_fp16_fp32" % (M, N, K), "value": value,
            "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 in, f32 accumulate/out",
            "data": "synthetic: seeded U[-1,1] fp16 generated on the device",
            "config": {"workload": "tensor-parallel K-split gemm %dx%dx%d, K slabs over N GPUs, "
                                   "partials reduce-scattered every step" % (M, N, K),
                       "reduce_scatter": ({"staged": "partials pushed to the peers' slots by "
                                                     "the copy engine during the next GEMM",
                                           "direct": "GEMMs store into the peers' slots",
                                           "fused": "GEMMs store into the peers' slots, own "
                                                    "slab's epilogue sums the slots"}[args.rs_form]
                                          + " (b2g_gemm_sharded_k_p2p)" if plan is not None
                                          else "ncclReduceScatter after the GEMM (b2g_gemm_sharded_k)"),
                       "p2p_form": args.rs_form if plan is not None else None,
                       "rows_per_rank": rows},
            "roofline": {"bound": "tensor" if t_gemm >= t_link else "nvlink",
                         "target_ms": target * 1e3, "frac": target * 1e3 / (ms / args.steps),
                         "gemm_ms_at_peak": t_gemm * 1e3, "nvlink_ms": t_link * 1e3,
                         "nvlink_bytes_per_rank": nv_bytes,
                         "peak_source": "%s bf16_tflops_sustained; peer copy 770 GB/s" % src},
            "row0_out_of_tolerance": bad, "device_status": status,
            "gpu_launches": launches}), flush=True)
    return 0


def graph_us_per_call(torch, fns, calls, replays=10):
    """Microseconds per call of each function in `fns`: `calls` calls of it captured in one CUDA
    graph, the graphs replayed in turn (A, B, A, B, ...) `replays` times, each replay between
    two events.  Device time with no host launch gaps (the host cost of a call, about 10 us
    through Python, hides small kernels otherwise); taking turns gives every function the same
    clocks under the power cap."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graphs = []
    for fn in fns:
        with torch.cuda.stream(s):
            for _ in range(3):
                fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(calls):
                fn()
        g.replay()
        torch.cuda.synchronize()
        graphs.append(g)
    total = [0.0] * len(fns)
    for _ in range(replays):
        for i, g in enumerate(graphs):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            total[i] += a.elapsed_time(b)
    del graphs
    return [t / (replays * calls) * 1000.0 for t in total]


def cublas_side_by_side(torch, dA, dB, dC, gpu, steps):
    """cuBLAS fp16 x fp16 -> fp32 on the same operands and box, after our timed region (a
    comparison only; the product path never calls it)."""
    try:
        out = torch.mm(dA, dB, out_dtype=torch.float32)
    except (TypeError, RuntimeError) as e:
        return {"unavailable": str(e).splitlines()[0][:120]}
    diff = float((out - dC).abs().max())
    for _ in range(5):
        torch.mm(dA, dB, out_dtype=torch.float32)
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu)
    sampler.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        torch.mm(dA, dB, out_dtype=torch.float32)
    t1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1) / steps
    M, K = dA.shape
    N = dB.shape[1]
    return {"value": 2.0 * M * N * K / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "steps": steps,
            "call": "torch.mm(A, B, out_dtype=torch.float32)", "clocks": clocks,
            "max_abs_diff_vs_b2g": diff}


def row_out_of_tolerance(torch, got_row, a_row, B, K):
    """Elements of one C row outside |C - R| <= 1e-3*sqrt(K)*max|a|*max|b| + 1e-3*|R|, R the
    FP64 PyTorch product of the same fp16 row and B (inputs in [-1, 1])."""
    ref = (a_row.to(torch.float64) @ B.to(torch.float64)).reshape(-1)
    got = got_row.to(device=ref.device, dtype=torch.float64).reshape(-1)
    tol = 1e-3 * K ** 0.5 + 1e-3 * ref.abs()
    return int(((got - ref).abs() > tol).sum().item() + torch.isnan(got).sum().item())


def e2e_run(torch, b2g, dev, M, N, K, rank, ws, steps, dist):
    """Pinned host A, B -> device, GEMM, C -> pinned host, every step.  Two buffer sets and
    three streams (H2D, compute, D2H) let step i+1's upload overlap step i's download."""
    # host inputs: the library's seeded generator, run once on the device and copied out
    gA = torch.empty((M, K), dtype=torch.float16, device=dev)
    gB = torch.empty((K, N), dtype=torch.float16, device=dev)
    b2g.fill_uniform(gA, M * K, 1, rank * M * K)
    b2g.fill_uniform(gB, K * N, 2)
    torch.cuda.synchronize()
    hA = gA.cpu().pin_memory()
    hB = gB.cpu().pin_memory()
    hC = [torch.empty((M, N), dtype=torch.float32).pin_memory() for _ in range(2)]
    bufs = [(torch.empty((M, K), dtype=torch.float16, device=dev),
             torch.empty((K, N), dtype=torch.float16, device=dev),
             torch.empty((M, N), dtype=torch.float32, device=dev)) for _ in range(2)]
    s_in, s_mm, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    up = [torch.cuda.Event() for _ in range(2)]
    mm = [torch.cuda.Event() for _ in range(2)]
    down = [torch.cuda.Event() for _ in range(2)]

    def run(n):
        for i in range(n):
            b = i & 1
            a_, b_, c_ = bufs[b]
            with torch.cuda.stream(s_in):
                s_in.wait_event(mm[b]) if i >= 2 else None
                a_.copy_(hA, non_blocking=True)
                b_.copy_(hB, non_blocking=True)
                up[b].record(s_in)
            s_mm.wait_event(up[b])
            if i >= 2:
                s_mm.wait_event(down[b])
            b2g.gemm(a_, b_, c_, M, N, K, K, N, N, s_mm)
            mm[b].record(s_mm)
            with torch.cuda.stream(s_out):
                s_out.wait_event(mm[b])
                hC[b].copy_(c_, non_blocking=True)
                down[b].record(s_out)

    run(2)
    torch.cuda.synchronize()
    link = pcie_bandwidth(torch, dev, hA, hB, hC[0], bufs[0])
    if dist is not None:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record(s_in)
    run(steps)
    s_in.wait_stream(s_out)
    t1.record(s_in)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # spot-check the result that came back (first row of the last step)
    bad = row_out_of_tolerance(torch, hC[(steps - 1) & 1][:1], gA[:1], gB, K)
    del gA, gB
    bi, bo = (M * K + K * N) * 2, M * N * 4
    # the copy bound of a step: its uploads and downloads at the pinned-copy bandwidths measured
    # above, the two directions overlapping (the GEMM runs under them)
    target_ms = max(bi / link["h2d_gbs"], bo / link["d2h_gbs"],
                    (bi + bo) / link["bidir_gbs"]) / 1e6
    roof = dict(link, bound="pcie", target_ms_per_step=target_ms,
                frac=target_ms / (ms / steps))
    return {"value": 2.0 * M * N * K * ws * steps / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
            "steps": steps, "ms_per_step": ms / steps, "row0_out_of_tolerance": bad,
            "pipeline": "2 buffer sets, H2D / compute / D2H streams", "roofline": roof}


def pcie_bandwidth(torch, dev, hA, hB, hC, dbuf):
    """Pinned host <-> device copy bandwidth of this GPU (GB/s, best of 3): uploads of A and B,
    a download of C, and both directions at once on two streams."""
    dA, dB, dC = dbuf
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def timed(fn):
        best = None
        for _ in range(3):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s1)
            s2.wait_event(e0)
            fn()
            s1.wait_stream(s2)
            e1.record(s1)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        return best

    def up():
        with torch.cuda.stream(s1):
            dA.copy_(hA, non_blocking=True)
            dB.copy_(hB, non_blocking=True)

    def down():
        with torch.cuda.stream(s2):
            hC.copy_(dC, non_blocking=True)

    bi = hA.numel() * hA.element_size() + hB.numel() * hB.element_size()
    bo = hC.numel() * hC.element_size()
    t_up, t_down = timed(up), timed(down)
    t_both = timed(lambda: (up(), down()))
    return {"h2d_gbs": bi / (t_up * 1e6), "d2h_gbs": bo / (t_down * 1e6),
            "bidir_gbs": (bi + bo) / (t_both * 1e6)}


if __name__ == "__main__":
    sys.exit(main())
