#!/usr/bin/env python3
"""Benchmark of the weight-only quantized linear hot path on B200.

Workload: GPTQ int4 W4A16 decode GEMMs, M in {1, 4, 8, 16},
K=5120, N=17408, group 128, asymmetric packed zeros, bf16 activations and
output, synthetic seeded data.  One step = the four GEMMs (one per M).  Every
GEMM of a run reads a different one of R weight copies in turn (R * 46 MB >
2 * L2), so weights stream from HBM.

Metric: algorithmic HBM bytes (qweight + scales + qzeros + A + C, each once)
per second.  With --gpus N every rank runs the same sweep on its own weights
(independent layers, no collective on the data path): weak scaling, value =
bytes of all ranks / max over ranks of the device time.

Output: one JSON line on rank 0 with ``value`` (device time, inputs resident
in HBM, steps replayed from CUDA graphs), ``e2e`` (the public API call with
pinned-host activations copied in and outputs copied out every step),
``roofline`` for the GEMV kernel (CUDA events per launch), ``cpu_baseline``
(the C oracle on the host cores) and ``clocks`` (nvidia-smi during the run).

``--impl reference`` times the reference's CPU path instead (the plain-C
restatement of its host loops; the reference's own SYCL code cannot be built
without icpx/oneAPI) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K, N, GS = 5120, 17408, 128
MS = (1, 4, 8, 16)
METRIC = json.load(open(os.path.join(ROOT, "BASELINE.json")))["metric"]
WORKLOAD = ("config2: GPTQ int4 W4A16 decode sweep, M in {1,4,8,16}, K=5120, N=17408, group 128, "
            "asymmetric packed zeros (v1 +1), bf16 activations and output, fp32 accumulate")
# dram__bytes_read.sum + dram__bytes_write.sum of one gptq_gemv launch at M=1 from the ncu
# capture summarised in profiles/gptq_gemv_config2.md (46.35 MB read + ~0.03 MB written).
TRAFFIC_PER_LAUNCH = 46_380_000


def alg_bytes(M: int, n_cols: int = N) -> int:
    qweight = K // 8 * n_cols * 4
    scales = K // GS * n_cols * 2
    qzeros = K // GS * n_cols // 8 * 4
    return qweight + scales + qzeros + M * K * 2 + M * n_cols * 2


def step_bytes(n_cols: int = N) -> int:
    return sum(alg_bytes(m, n_cols) for m in MS)


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy burst)"
    return 6650.0, "fallback (6.65 TB/s pool measurement)"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f".clocks_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.remove(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        power = [num(r[3]) for r in rows if num(r[3]) is not None]
        load = [s for s, p in zip(sm, power) if p is not None and p > 0.3 * max(power)] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": num(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(power) if power else None}


# ----------------------------------------------------------------------------- CPU side
def cpu_sweep(weights_np, acts_np, threads: int = 0) -> float:
    """One pass of the reference CPU path (oracle restatement) over the sweep; returns seconds."""
    import oracle as O
    qw, qz, sc = weights_np
    n_cols = qw.shape[1]
    t0 = time.perf_counter()
    for M in MS:
        O.gptq_gemm(acts_np[M], qw, qz, sc, None, M, n_cols, K, GS, 1, threads=threads)
    return time.perf_counter() - t0


def cpu_weights(seed: int, n_cols: int):
    import numpy as np
    rng = np.random.default_rng(seed)
    qw = rng.integers(-2**31, 2**31, size=(K // 8, n_cols), dtype=np.int64).astype(np.int32)
    qz = rng.integers(-2**31, 2**31, size=(K // GS, n_cols // 8), dtype=np.int64).astype(np.int32)
    sc = (np.abs(rng.standard_normal((K // GS, n_cols))) * 0.02 + 1e-3).astype(np.float16).view(np.uint16)
    acts = {M: rng.standard_normal((M, K)).astype(np.float32) for M in MS}
    return (qw, qz, np.ascontiguousarray(sc)), acts


def _sample_columns(seconds_per_sweep: float, cores: int) -> int:
    """Columns of the sweep whose oracle pass takes about ``seconds_per_sweep``."""
    w, a = cpu_weights(0, 1024)
    cpu_sweep(w, a, cores)
    t1 = cpu_sweep(w, a, cores)
    return int(min(N, max(64, 1024 * seconds_per_sweep / max(t1, 1e-6))) // 64 * 64)


def cpu_baseline(target_s: float = 12.0) -> dict:
    """Time the oracle on a bounded sample: whole sweeps on a column subset, all host cores."""
    cores = os.cpu_count() or 1
    n_cols = _sample_columns(target_s / 3, cores)
    weights, acts = cpu_weights(0, n_cols)
    reps, total, nbytes = 0, 0.0, 0
    while total < target_s and reps < 200:
        total += cpu_sweep(weights, acts, cores)
        nbytes += step_bytes(n_cols)
        reps += 1
    return {"value": round(nbytes / total / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{reps} full M-sweep(s) on {n_cols} of {N} columns (oracle/w4_oracle.c orc_gptq_gemm, "
                      f"OpenMP {cores} threads)",
            "seconds": round(total, 3)}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    O.build()
    cores = os.cpu_count() or 1
    budget = 60.0 / max(1, args.steps + args.warmup)  # whole run within about a minute
    n_cols = _sample_columns(budget, cores)
    weights, acts = cpu_weights(0, n_cols)
    for _ in range(args.warmup):
        cpu_sweep(weights, acts, cores)
    times = [cpu_sweep(weights, acts, cores) for _ in range(args.steps)]
    total = sum(times)
    value = step_bytes(n_cols) * args.steps / total / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_columns": n_cols},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"each step: the M-sweep on {n_cols} of {N} columns; the reference's SYCL "
                                   "host code needs icpx (absent), so its loops run as the plain-C oracle"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU side
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from xe2x2_b200 import ops, synth
    from xe2x2_b200 import _lib as L

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    L.lib()

    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 2**20) or 126 * 2**20
    wbytes = alg_bytes(0)
    R = max(4, math.ceil(2 * l2 / wbytes) + 1)
    weights = [synth.gptq_weights(K, N, GS, asym=True, seed=1000 * rank + r, device=dev)[:3] for r in range(R)]
    acts = {M: synth.activations(M, K, torch.bfloat16, seed=M, device=dev) for M in MS}
    outs = {M: torch.empty((M, N), dtype=torch.bfloat16, device=dev) for M in MS}
    period = R // math.gcd(len(MS), R)

    def gemm(M, w, out):
        qw, qz, sc = w
        L.call("w4_gptq_gemm", ops._p(acts[M]), L.W4_BF16, ops._p(qw), ops._p(qz), ops._p(sc), None,
               ops._p(out), L.W4_BF16, None, M, N, K, GS, 1, None, 0, ops._stream(dev))

    def step(i):
        for j, M in enumerate(MS):
            gemm(M, weights[(len(MS) * i + j) % R], outs[M])

    # warm up eagerly (first launches load modules), then capture one graph per rotation phase
    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    graphs = []
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        for ph in range(period):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                step(ph)
            graphs.append(g)
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-resident timed region
    for i in range(args.warmup):
        graphs[i % period].replay()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(args.steps):
        graphs[i % period].replay()
    e1.record(st)
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    value = step_bytes() * args.steps * world / (ms / 1e3) / 1e9

    # ---------------- per-launch kernel durations (roofline of the GEMV kernel):
    # for each M, launches over the rotating weights captured back to back in one
    # graph; CUDA events around its replays give the mean launch duration.
    from xe2x2_b200.profile_driver import time_graph
    per_m = {}
    for M in MS:
        us = time_graph(lambda r, M=M: gemm(M, weights[r % R], outs[M]), max(30, 2 * R))
        per_m[str(M)] = {"us": round(us, 3), "GB/s": round(alg_bytes(M) / us / 1e3, 1)}
    tot_b = sum(alg_bytes(M) for M in MS)
    tot_us = sum(per_m[str(M)]["us"] for M in MS)
    achieved = tot_b / tot_us / 1e3
    peak, peak_src = measured_peak()

    # ---------------- end to end through the public API (pinned host in, host out)
    # Each step's inputs (the four activation blocks) travel from pinned host memory
    # in one copy and its four outputs come back in one, as a serving loop runs them:
    # copies on their own streams, double-buffered, so step t+1's upload and step
    # t-1's download overlap step t's GEMMs.  G steps (a whole number of weight
    # rotations and of buffer pairs) are captured in one multi-stream graph.
    rows = sum(MS)
    NB = 2
    h_in = [torch.cat([acts[M].cpu() for M in MS]).pin_memory() for _ in range(NB)]
    h_out = [torch.empty((rows, N), dtype=torch.bfloat16).pin_memory() for _ in range(NB)]
    d_in = [torch.empty((rows, K), dtype=torch.bfloat16, device=dev) for _ in range(NB)]
    d_out = [torch.empty((rows, N), dtype=torch.bfloat16, device=dev) for _ in range(NB)]
    offs = [sum(MS[:j]) for j in range(len(MS))]
    G = period * NB // math.gcd(period, NB)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = {k: [torch.cuda.Event() for _ in range(G)] for k in ("in", "comp", "out")}

    def e2e_steps():
        fork = torch.cuda.Event()
        fork.record(cap)
        s_in.wait_event(fork)
        s_out.wait_event(fork)
        for t in range(G):
            p = t % NB
            with torch.cuda.stream(s_in):
                if t >= NB:
                    s_in.wait_event(ev["comp"][t - NB])  # d_in[p] read by step t - NB
                d_in[p].copy_(h_in[p], non_blocking=True)
                ev["in"][t].record(s_in)
            cap.wait_event(ev["in"][t])
            if t >= NB:
                cap.wait_event(ev["out"][t - NB])  # d_out[p] downloaded by step t - NB
            for j, M in enumerate(MS):
                qw, qz, sc = weights[(len(MS) * t + j) % R]
                ops.gptq_gemm(d_in[p][offs[j]:offs[j] + M], qw, qz, sc, GS, 1, out=d_out[p][offs[j]:offs[j] + M])
            ev["comp"][t].record(cap)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev["comp"][t])
                h_out[p].copy_(d_out[p], non_blocking=True)
                ev["out"][t].record(s_out)
        cap.wait_event(ev["out"][G - 1])
        cap.wait_event(ev["in"][G - 1])

    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        e2e_steps()  # eager pass: modules loaded, workspaces sized
    torch.cuda.synchronize()
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g_e2e, stream=cap):
            e2e_steps()
    torch.cuda.synchronize()
    # the pipeline's last output against a direct call
    pl = (G - 1) % NB
    g_e2e.replay()
    torch.cuda.synchronize()
    for j, M in enumerate(MS):
        qw, qz, sc = weights[(len(MS) * (G - 1) + j) % R]
        want = ops.gptq_gemm(acts[M], qw, qz, sc, GS, 1)
        if not torch.equal(h_out[pl][offs[j]:offs[j] + M], want.cpu()):
            raise RuntimeError(f"end-to-end pipeline output differs from the direct call at M={M}")
    reps = max(1, -(-args.steps // G))
    for i in range(max(1, -(-args.warmup // G))):
        g_e2e.replay()
    barrier()
    e0.record(st)
    for i in range(reps):
        g_e2e.replay()
    e1.record(st)
    barrier()
    e2e_steps_done = reps * G
    ms_e2e = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = step_bytes() * e2e_steps_done * world / (ms_e2e / 1e3) / 1e9
    h2d = sum(M * K * 2 for M in MS)
    d2h = sum(M * N * 2 for M in MS)

    cpu = cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None

    # release graphs before the process group goes away
    graphs.clear()
    del g_e2e
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "step": "4 GEMMs (M=1,4,8,16) replayed from a CUDA graph",
                       "l2": f"inputs larger than L2: weights rotate over {R} copies "
                             f"({R * wbytes / 1e6:.0f} MB vs {l2 / 1e6:.0f} MB L2)",
                       "parallelism": f"{world} independent replicas (no data-path collective)",
                       "algorithmic_bytes_per_step": step_bytes()},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "path": "ops.gptq_gemm per M; each step's activations in one pinned-host copy and its outputs "
                            "out in one, on separate streams with double buffers so copies overlap the neighbouring "
                            f"steps' GEMMs; {G}-step multi-stream graph replayed",
                    "steps": e2e_steps_done, "ms_per_step": round(ms_e2e / e2e_steps_done, 5)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": TRAFFIC_PER_LAUNCH,
                         "kernel": "w4::gptq_gemv_tma_kernel", "peak_source": peak_src,
                         "per_m": per_m},
            "gpu_launches": len(MS) * args.steps,
            "clocks": clk,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- TP layer set
TP_MS = (1, 32, 256)
TP_WORKLOAD = ("config5: one 27B-class dense layer's GPTQ g128 projections (QKV N=7168 and gate|up N=34816 "
               "column-parallel, o 5120x5120 and down K=17408 row-parallel with an NCCL all-reduce of bf16 "
               "outputs), M in {1,32,256}, tensor-parallel over the ranks, attention math excluded")


def run_tp(args) -> None:
    """Tensor-parallel layer set (config 5) at TP = number of ranks: strong scaling."""
    import torch
    import torch.distributed as dist

    from xe2x2_b200 import _lib as L
    from xe2x2_b200 import tp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    def trace(msg):
        if args.trace:
            print(f"[rank {rank}] {time.strftime('%H:%M:%S')} {msg}", file=sys.stderr, flush=True)

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    L.lib()
    trace("process group up")
    comm = tp.TPComm(rank, world, timeout_ms=120000, device=dev)
    trace("communicator up")
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 2**20) or 126 * 2**20
    sets = [tp.TPLayerSet(comm, rank, world, dev, seed=0)]
    per_rank = sets[0].weight_bytes_per_rank()
    R = max(2, math.ceil(2 * l2 / per_rank) + 1)
    sets += [tp.TPLayerSet(comm, rank, world, dev, seed=1000 * r) for r in range(1, R)]
    xs = {M: sets[0].inputs(M) for M in TP_MS}
    outs = {M: {p.name: torch.empty((M, p.N // world if p.mode == "column" else p.N), dtype=torch.bfloat16,
                                     device=dev) for p in sets[0].projs} for M in TP_MS}

    def step(i):
        for j, M in enumerate(TP_MS):
            sets[(len(TP_MS) * i + j) % R].step(xs[M], outs[M])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    period = R // math.gcd(len(TP_MS), R)
    trace(f"{R} layer sets built")
    for i in range(3):
        step(i)
    comm.wait()
    barrier()
    trace("eager warm-up done")
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    graphs = []
    with torch.cuda.stream(cap):
        for ph in range(period):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                step(ph)
            graphs.append(g)
    torch.cuda.current_stream().wait_stream(cap)
    barrier()
    trace("graphs captured")
    for i in range(args.warmup):
        graphs[i % period].replay()
    comm.wait()
    trace("graph warm-up done")
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(args.steps):
        graphs[i % period].replay()
    e1.record(st)
    trace("timed steps enqueued")
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    trace(f"timed region: {ms:.3f} ms")

    # per-M layer time and all-reduce time alone (graphs of one M / of the bare collectives)
    per_m = {}
    for M in TP_MS:
        gm = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(gm, stream=cap):
                for r in range(R):
                    sets[r].step(xs[M], outs[M])
        torch.cuda.current_stream().wait_stream(cap)
        trace(f"M={M}: layer graph captured")
        ga = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(ga, stream=cap):
                for r in range(R):
                    comm.allreduce_(outs[M]["o"])
                    comm.allreduce_(outs[M]["down"])
        torch.cuda.current_stream().wait_stream(cap)
        # decode sizes at TP > 1: the same layer with the row-parallel GEMMs reducing in
        # their own epilogue (the default is GEMM + one-shot all-reduce)
        gu = None
        if world > 1 and M <= 16:
            comm.set_fused_epilogue(True)
            gu = torch.cuda.CUDAGraph()
            with torch.cuda.stream(cap):
                with torch.cuda.graph(gu, stream=cap):
                    for r in range(R):
                        sets[r].step(xs[M], outs[M])
            torch.cuda.current_stream().wait_stream(cap)
            comm.set_fused_epilogue(False)
        res = []
        for g in (gm, ga) + ((gu,) if gu is not None else ()):
            for _ in range(3):
                g.replay()
            barrier()
            e0.record(st)
            for _ in range(5):
                g.replay()
            e1.record(st)
            barrier()
            res.append(max_over_ranks(e0.elapsed_time(e1)) * 1e3 / (5 * R))
            trace(f"M={M}: {res[-1]:.2f} us")
        per_m[str(M)] = {"layer_us": round(res[0], 2), "allreduce_us": round(res[1], 2),
                         "TFLOP/s": round(sets[0].flops(M) / res[0] / 1e6, 2)}
        if gu is not None:
            per_m[str(M)]["layer_fused_epilogue_us"] = round(res[2], 2)
        del gm, ga, gu, g  # graphs holding NCCL work must be gone before the communicator is
    graphs.clear()
    torch.cuda.synchronize()
    comm.close()

    full_w = sum(p.K // 8 * p.N * 4 + p.K // 128 * p.N * 2 + p.K // 128 * p.N // 8 * 4 for p in sets[0].projs)
    step_bytes_tp = sum(full_w + sum(M * p.K * 2 + M * p.N * 2 for p in sets[0].projs) for M in TP_MS)
    value = step_bytes_tp * args.steps / (ms / 1e3) / 1e9
    peak, peak_src = measured_peak()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": TP_WORKLOAD, "parallelism": f"tp{world}",
                       "step": "12 GEMMs + 6 all-reduces (4 projections x M=1,32,256) replayed from a CUDA graph",
                       "l2": f"inputs larger than L2: {R} layer-set copies of {per_rank / 1e6:.1f} MB per rank",
                       "algorithmic_bytes_per_step": step_bytes_tp,
                       "flops_per_step": sum(sets[0].flops(M) for M in TP_MS)},
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": round(peak * world, 1),
                         "unit": "GB/s", "frac": round(value / (peak * world), 4), "traffic": None,
                         "peak_source": f"{world} x {peak_src}", "per_m": per_m},
            "gpu_launches": None, "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--trace", action="store_true", help="progress lines on stderr")
    ap.add_argument("--workload", choices=["decode", "tp"], default="decode",
                    help="decode: config 2 sweep (default); tp: config 5 layer set at TP = --gpus")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "tp":
        run_tp(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
