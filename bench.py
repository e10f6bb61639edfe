#!/usr/bin/env python3
"""Benchmark of the weight-only quantized linear hot path on B200.

One GPU (``--gpus 1``, the default): BASELINE config 2 -- GPTQ int4 W4A16 decode GEMMs,
M in {1, 4, 8, 16}, K=5120, N=17408, group 128, asymmetric packed zeros, bf16 activations
and output, synthetic seeded data.  Every GEMM reads a different one of R weight copies in
turn (R * 46 MB > 2 * L2), so weights stream from HBM.  A step is three rotations over the R
copies of the M-sweep (3 * 4 * R GEMMs), replayed from CUDA graphs.  Metric: algorithmic HBM
bytes (qweight + scales + qzeros + A + C, each once) per second.  The same line carries
``per_config``: configs 1, 3 and 4 (GPTQ M=16 4096^2 f16; NVFP4 5120^2 M=1..8192 with bf16
or NVFP4 activations; GPTQ act_order prefill M=2048/8192), each timed on the device with its
roofline fraction and the CPU oracle timed beside it on a bounded sample; ``moe``: the grouped
(MoE) GEMMs over 8 experts of hidden 2688 x expert 1856; and ``tp1``: the config 5 layer set at
TP=1.

Several GPUs (``--gpus N`` under torchrun): BASELINE config 5 -- one 27B-class layer's GPTQ
projections (QKV and gate|up column-parallel, o and down row-parallel with the all-reduce of
their bf16 outputs), M in {1, 32, 256}, tensor-parallel over the N ranks (strong scaling:
the same layer whatever N).  ``--workload replicas`` runs N independent copies of config 2
instead (weak scaling, no collective).

Output: one JSON line on rank 0 with ``value`` (device time, inputs resident in HBM),
``e2e`` (the public API with every step's activations copied in from pinned host memory and
its outputs copied out), ``roofline`` for the dominant kernel (with ``read_ceiling``: the read
bandwidth a plain one-launch read of the same bytes attains, timed the same way), ``cpu_baseline`` (the C oracle
on the host cores) and ``clocks`` (nvidia-smi during the timed region).

``--impl reference`` times the reference's CPU path instead (the plain-C restatement of its
host loops; the reference's own SYCL code cannot be built without icpx/oneAPI) on a bounded
sample of the same workload, with the same ``config`` keys.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import platform
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K, N, GS = 5120, 17408, 128
MS = (1, 4, 8, 16)
ROTATIONS_PER_STEP = 3
METRIC = json.load(open(os.path.join(ROOT, "BASELINE.json")))["metric"]
WORKLOAD = ("config2: GPTQ int4 W4A16 decode sweep, M in {1,4,8,16}, K=5120, N=17408, group 128, "
            "asymmetric packed zeros (v1 +1), bf16 activations and output, fp32 accumulate")
# dram__bytes_read.sum + dram__bytes_write.sum of one config 2 decode launch at M=1 (ncu capture of the
# decode kernel: 46,365,952 read + 13,312 written; the algorithmic bytes are 46.35 MB).
TRAFFIC_PER_LAUNCH = 46_379_264


def alg_bytes(M: int, n_cols: int = N, k: int = K) -> int:
    qweight = k // 8 * n_cols * 4
    scales = k // GS * n_cols * 2
    qzeros = k // GS * n_cols // 8 * 4
    return qweight + scales + qzeros + M * k * 2 + M * n_cols * 2


def sweep_bytes(n_cols: int = N) -> int:
    return sum(alg_bytes(m, n_cols) for m in MS)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm": float(d["hbm_gbs"]), "bf16": float(d["bf16_tflops"]),
                "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback (earlier pool measurement)"}


FP4_NOMINAL_TFLOPS = 9000.0  # dense FP4, datasheet: no measured FP4 peak on this pool


def cpu_info() -> dict:
    model = platform.processor() or ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_model": model, "cpu_threads": os.cpu_count() or 1}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix="w4_clocks_", suffix=".csv")
        os.close(fd)

    def start(self):
        try:
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


# ----------------------------------------------------------------------------- device timing
def time_graph(fn, reps: int) -> float:
    """Mean device time (us) of one ``fn(i)``: ``reps`` calls captured in one CUDA graph, the graph
    replayed 5 times between CUDA events on the current stream (no host work between launches)."""
    import torch
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        for r in range(3):
            fn(r)
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for r in range(reps):
            fn(r)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (5 * reps)


def graph_kernels(graph) -> dict | None:
    """Kernel nodes of a captured CUDA graph (torch ``CUDAGraph(keep_graph=True)``) by origin:
    ``w4`` (this library's kernels: mangled names in namespace w4), ``nccl`` and ``other``, with
    the names of the ``other`` ones.  None when the graph cannot be inspected (cuda-python missing
    or an unexpected driver)."""
    try:
        from cuda.bindings import driver as drv
        g = drv.CUgraph(graph.raw_cuda_graph())
        err, _, n = drv.cuGraphGetNodes(g, 0)
        if err != drv.CUresult.CUDA_SUCCESS:
            return None
        err, nodes, n = drv.cuGraphGetNodes(g, n)
        counts = {"w4": 0, "nccl": 0, "other": 0}
        others = set()
        for nd in nodes[:n]:
            err, t = drv.cuGraphNodeGetType(nd)
            if err != drv.CUresult.CUDA_SUCCESS or t != drv.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
                continue
            err, prm = drv.cuGraphKernelNodeGetParams(nd)
            if err != drv.CUresult.CUDA_SUCCESS:
                return None
            name = b""
            fn, kern = getattr(prm, "func", None), getattr(prm, "kern", None)
            if fn is not None and int(fn):
                err, name = drv.cuFuncGetName(fn)
            elif kern is not None and int(kern):
                err, name = drv.cuKernelGetName(kern)
            if err != drv.CUresult.CUDA_SUCCESS or not name:
                return None
            name = name.decode() if isinstance(name, bytes) else str(name)
            key = "w4" if "2w4" in name[:12] else ("nccl" if "nccl" in name[:24] else "other")
            counts[key] += 1
            if key == "other":
                others.add(name[:120])
        if others:
            counts["other_names"] = sorted(others)
        return counts
    except Exception:  # noqa: BLE001 - introspection is best effort; the caller reports None
        return None


def copies_for(nbytes: int, l2: int) -> int:
    """Weight copies that together exceed twice the L2 (every launch then reads HBM)."""
    return max(2, math.ceil(2 * l2 / max(nbytes, 1)) + 1)


# ----------------------------------------------------------------------------- CPU side
def _gptq_np(seed: int, k: int, n_cols: int, asym: bool = True):
    import numpy as np
    rng = np.random.default_rng(seed)
    qw = rng.integers(-2**31, 2**31, size=(k // 8, n_cols), dtype=np.int64).astype(np.int32)
    qz = rng.integers(-2**31, 2**31, size=(k // GS, n_cols // 8), dtype=np.int64).astype(np.int32) if asym else None
    sc = (np.abs(rng.standard_normal((k // GS, n_cols))) * 0.02 + 1e-3).astype(np.float16).view(np.uint16)
    return qw, qz, np.ascontiguousarray(sc)


def cpu_sweep(weights_np, acts_np, threads: int) -> float:
    """One pass of the reference CPU path (oracle restatement) over the M-sweep; returns seconds."""
    import oracle as O
    qw, qz, sc = weights_np
    n_cols = qw.shape[1]
    t0 = time.perf_counter()
    for M in MS:
        O.gptq_gemm(acts_np[M], qw, qz, sc, None, M, n_cols, K, GS, 1, threads=threads)
    return time.perf_counter() - t0


def cpu_sweep_inputs(seed: int, n_cols: int):
    import numpy as np
    rng = np.random.default_rng(seed + 1)
    return _gptq_np(seed, K, n_cols), {M: rng.standard_normal((M, K)).astype(np.float32) for M in MS}


def sample_columns(seconds: float, threads: int) -> int:
    """Columns of the sweep whose oracle pass takes about ``seconds``."""
    w, a = cpu_sweep_inputs(0, 512)
    cpu_sweep(w, a, threads)
    t1 = cpu_sweep(w, a, threads)
    return int(min(N, max(64, 512 * seconds / max(t1, 1e-6))) // 64 * 64)


def cpu_baseline(target_s: float = 10.0) -> dict:
    """The oracle on bounded samples of the config 2 sweep: all host cores, and one core (the
    reference's loop order, single thread)."""
    cores = os.cpu_count() or 1
    out = {}
    for label, threads, budget in (("all_cores", cores, target_s), ("single_thread", 1, target_s / 3)):
        n_cols = sample_columns(budget / 3, threads)
        weights, acts = cpu_sweep_inputs(0, n_cols)
        reps, total, nbytes = 0, 0.0, 0
        while total < budget and reps < 200:
            total += cpu_sweep(weights, acts, threads)
            nbytes += sweep_bytes(n_cols)
            reps += 1
        out[label] = {"value": round(nbytes / total / 1e9, 4), "unit": "GB/s", "threads": threads,
                      "sample": f"{reps} M-sweep(s) on {n_cols} of {N} columns", "seconds": round(total, 3)}
    line = {"value": out["all_cores"]["value"], "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": out["all_cores"]["sample"] + " (oracle/w4_oracle.c orc_gptq_gemm, OpenMP)",
            "single_thread": out["single_thread"]}
    line.update(cpu_info())
    return line


def cpu_rate(fn, flops_per_call: float, bytes_per_call: float, budget_s: float) -> dict:
    """Repeat ``fn`` (an oracle call on a sample) for about ``budget_s`` seconds."""
    reps, total = 0, 0.0
    while total < budget_s and reps < 1000:
        t0 = time.perf_counter()
        fn()
        total += time.perf_counter() - t0
        reps += 1
    return {"seconds_per_call": total / reps, "GFLOP/s": round(flops_per_call * reps / total / 1e9, 3),
            "GB/s": round(bytes_per_call * reps / total / 1e9, 4), "calls": reps}


# ----------------------------------------------------------------------------- per-config measurements
def per_config(dev, pk, cpu: bool) -> dict:
    """Configs 1, 3 and 4 of BASELINE.json: device time per launch (CUDA graph of launches over
    weights rotated past 2x L2), the roofline fraction, and the oracle on a bounded CPU sample."""
    import numpy as np
    import torch

    import oracle as O
    from xe2x2_b200 import _lib as L
    from xe2x2_b200 import ops, synth

    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    cores = os.cpu_count() or 1
    res = {}

    # config 1: GPTQ M=16, K=N=4096, g128, symmetric (stored zero 7, v1), f16 in/out
    k1 = n1 = 4096
    wb = k1 // 8 * n1 * 4 + k1 // GS * n1 * 2
    R = copies_for(wb, l2)
    ws = [synth.gptq_weights(k1, n1, GS, asym=False, seed=10 + r, device=dev) for r in range(R)]
    a = synth.activations(16, k1, torch.float16, seed=1, device=dev)
    us = time_graph(lambda r: ops.gptq_gemm(a, ws[r % R][0], None, ws[r % R][2], GS, 1), max(2 * R, 20))
    nb = wb + 16 * k1 * 2 + 16 * n1 * 2
    c1 = {"shape": "M=16 K=N=4096 g128 sym f16", "us": round(us, 3), "GB/s": round(nb / us / 1e3, 1),
          "bound": "hbm", "frac": round(nb / us / 1e3 / pk["hbm"], 4), "algorithmic_bytes": nb}
    if cpu:
        qw, _, sc = _gptq_np(3, k1, n1, asym=False)
        an = np.random.default_rng(4).standard_normal((16, k1)).astype(np.float32)
        r_all = cpu_rate(lambda: O.gptq_gemm(an, qw, None, sc, None, 16, n1, k1, GS, 1, threads=cores),
                         2 * 16 * n1 * k1, nb, 2.0)
        qw1, sc1 = np.ascontiguousarray(qw[:, :512]), np.ascontiguousarray(sc[:, :512])
        r_one = cpu_rate(lambda: O.gptq_gemm(an, qw1, None, sc1, None, 16, 512, k1, GS, 1, threads=1),
                         2 * 16 * 512 * k1, nb * 512 / n1, 1.0)
        c1["cpu_baseline"] = {"GB/s": r_all["GB/s"], "cores": cores, "kind": "port", "sample": "full shape",
                              "single_thread_GB/s": r_one["GB/s"], "single_thread_sample": "512 of 4096 columns"}
    res["config1"] = c1
    del ws

    # config 3: NVFP4 K=N=5120; bf16 activations (the external operator's W4A16 form) and NVFP4
    # activations quantised in the call (block-scaled FP4 tensor cores)
    k3 = n3 = 5120
    wb = n3 * k3 // 2 + k3 // 16 * n3 + 4
    R = copies_for(wb, l2)
    ws = [synth.nvfp4_weights(k3, n3, seed=20 + r, device=dev) for r in range(R)]
    c3 = {"shape": "NVFP4 K=N=5120, e4m3 block scales g16, fp32 tensor scale, bf16 out", "w4a16": {},
          "nvfp4_act": {}}
    for M in (1, 16, 128, 2048, 8192):
        a = synth.activations(M, k3, torch.bfloat16, seed=M, device=dev)
        ag = torch.tensor([float(a.float().abs().max()) / (448.0 * 6.0)], dtype=torch.float32, device=dev)
        nb = wb + M * k3 * 2 + M * n3 * 2
        fl = 2.0 * M * n3 * k3
        reps = max(R, 20) if M <= 128 else max(R, 6)
        us = time_graph(lambda r: ops.nvfp4_gemm(a, ws[r % R][0], ws[r % R][1], ws[r % R][2]), reps)
        hbm = M <= 128
        c3["w4a16"][str(M)] = {"us": round(us, 3), "GB/s": round(nb / us / 1e3, 1),
                               "TFLOP/s": round(fl / us / 1e6, 2), "bound": "hbm" if hbm else "tensor(bf16)",
                               "frac": round(nb / us / 1e3 / pk["hbm"], 4) if hbm else round(fl / us / 1e6 / pk["bf16"], 4)}
        if M >= 128:
            us = time_graph(lambda r: ops.nvfp4_gemm(a, ws[r % R][0], ws[r % R][1], ws[r % R][2],
                                                     act_mode=L.W4_ACT_NVFP4, a_global=ag), reps)
            c3["nvfp4_act"][str(M)] = {"us": round(us, 3), "TFLOP/s": round(fl / us / 1e6, 2), "GB/s": round(nb / us / 1e3, 1),
                                       "bound": "hbm" if M == 128 else "tensor(fp4)",
                                       "frac": round(nb / us / 1e3 / pk["hbm"], 4) if M == 128
                                       else round(fl / us / 1e6 / FP4_NOMINAL_TFLOPS, 4),
                                       "includes": "activation quantiser + block-scaled GEMM"}
    if cpu:
        w_nk = np.random.default_rng(5).integers(0, 256, (512, k3 // 2), dtype=np.uint8)
        sc = torch.exp2(torch.rand((k3 // 16, 512)) * 8 - 6).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        an = np.random.default_rng(6).standard_normal((16, k3)).astype(np.float32)
        fl = 2.0 * 16 * 512 * k3
        r_all = cpu_rate(lambda: O.nvfp4_gemm(an, w_nk, 1, sc, 0, 1.0 / 448, 16, 512, k3, threads=cores), fl,
                         512 * k3 // 2 + k3 // 16 * 512, 2.0)
        r_one = cpu_rate(lambda: O.nvfp4_gemm(an, w_nk, 1, sc, 0, 1.0 / 448, 16, 512, k3, threads=1), fl,
                         512 * k3 // 2 + k3 // 16 * 512, 1.0)
        c3["cpu_baseline"] = {"GFLOP/s": r_all["GFLOP/s"], "cores": cores, "single_thread_GFLOP/s": r_one["GFLOP/s"],
                              "kind": "port", "sample": "M=16 x 512 of 5120 columns (orc_nvfp4_gemm); the rate scales "
                                                        "linearly to the other M"}
    res["config3"] = c3
    del ws

    # config 4: GPTQ act_order prefill, K=5120, N=27648, g128, asymmetric, bf16
    k4, n4 = 5120, 27648
    wb = k4 // 8 * n4 * 4 + k4 // GS * n4 * 2 + k4 // GS * n4 // 8 * 4 + k4 * 4
    R = copies_for(wb, l2)
    lins = []
    for r in range(R):
        qw, qz, sc, gi = synth.gptq_weights(k4, n4, GS, asym=True, seed=30 + r, device=dev, act_order=True)
        lins.append(ops.GPTQLinear(qw, qz, sc, gi, GS, 1))
    c4 = {"shape": "act_order K=5120 N=27648 g128 asym bf16"}
    for M in (2048, 8192):
        a = synth.activations(M, k4, torch.bfloat16, sigma=0.5, seed=M, device=dev)
        us = time_graph(lambda r: lins[r % R](a), max(R, 4))
        fl = 2.0 * M * n4 * k4
        c4[str(M)] = {"us": round(us, 2), "TFLOP/s": round(fl / us / 1e6, 1), "bound": "tensor(bf16)",
                      "frac": round(fl / us / 1e6 / pk["bf16"], 4), "frac_of": "bf16 burst"}
    if cpu:
        qw, qz, sc = _gptq_np(7, k4, n4)
        perm = np.random.default_rng(8).permutation(k4)
        gi = np.empty(k4, np.int32)
        gi[perm] = np.arange(k4, dtype=np.int32) // GS
        rows = 16
        an = np.random.default_rng(9).standard_normal((rows, k4)).astype(np.float32) * 0.5
        fl = 2.0 * rows * n4 * k4
        r_all = cpu_rate(lambda: O.gptq_gemm(an, qw, qz, sc, gi, rows, n4, k4, GS, 1, threads=cores), fl, 0, 3.0)
        qw1, qz1, sc1 = (np.ascontiguousarray(x) for x in (qw[:, :1024], qz[:, :128], sc[:, :1024]))
        r_one = cpu_rate(lambda: O.gptq_gemm(an, qw1, qz1, sc1, gi, rows, 1024, k4, GS, 1, threads=1),
                         2.0 * rows * 1024 * k4, 0, 1.5)
        c4["cpu_baseline"] = {"GFLOP/s": r_all["GFLOP/s"], "cores": cores, "kind": "port",
                              "single_thread_GFLOP/s": r_one["GFLOP/s"],
                              "sample": f"{rows} rows x all 27648 columns (all cores), {rows} rows x 1024 columns "
                                        "(one core); M=2048 / 8192 scale linearly",
                              "est_s_M2048": round(2.0 * 2048 * n4 * k4 / (r_all["GFLOP/s"] * 1e9), 1)}
    res["config4"] = c4
    del lins
    torch.cuda.empty_cache()
    res["moe"] = moe_record(dev, pk, l2)
    return res


MOE_COUNTS = {"decode_top6": [1, 1, 0, 1, 1, 1, 0, 1], "batch32_top6": [24, 31, 0, 17, 40, 29, 33, 18]}


def moe_record(dev, pk, l2) -> dict:
    """Grouped (MoE) GEMMs, one launch over 8 experts of hidden 2688 x expert 1856 (the
    reference's Lightning MoE shapes): GPTQ g128 and NVFP4, up (K=2688, N=1856) and down (K=1856,
    N=2688, GPTQ g64), ragged token counts.  Bytes: the weights of the experts with tokens."""
    import torch

    from xe2x2_b200 import ops, synth
    H, X, E = 2688, 1856, 8
    out = {"shape": "8 experts, hidden 2688 x expert 1856", "counts": MOE_COUNTS}
    for proj, K, N, gs in (("up", H, X, 128), ("down", X, H, 64)):
        wb1 = K // 8 * N * 4 + K // gs * N * 2 + K // gs * N // 8 * 4
        R = copies_for(wb1 * E, l2)
        gq = []
        for r in range(R):
            ws = [synth.gptq_weights(K, N, gs, asym=True, seed=100 * r + e, device=dev)[:3] for e in range(E)]
            gq.append(tuple(torch.stack([w[i] for w in ws]).contiguous() for i in range(3)))
        fb1 = N * K // 2 + K // 16 * N
        fq = []
        for r in range(copies_for(fb1 * E, l2)):
            ws = [synth.nvfp4_weights(K, N, seed=100 * r + e, device=dev) for e in range(E)]
            fq.append((torch.stack([w[0].t() for w in ws]).contiguous(), torch.stack([w[1] for w in ws]).contiguous(),
                       torch.cat([w[2] for w in ws]).contiguous()))
        for name, cnt in MOE_COUNTS.items():
            off = [0]
            for c in cnt:
                off.append(off[-1] + c)
            active = sum(1 for c in cnt if c)
            a = synth.activations(off[-1], K, torch.bfloat16, seed=1, device=dev)
            us = time_graph(lambda r: ops.gptq_gemm_grouped(a, *gq[r % len(gq)], off, gs, 1), max(2 * len(gq), 20))
            nb = active * wb1 + off[-1] * (K + N) * 2
            out[f"gptq_{proj}_{name}"] = {"us": round(us, 2), "GB/s": round(nb / us / 1e3, 1),
                                          "frac": round(nb / us / 1e3 / pk["hbm"], 4)}
            us = time_graph(lambda r: ops.nvfp4_gemm_grouped(a, *fq[r % len(fq)], off), max(2 * len(fq), 20))
            nb = active * fb1 + off[-1] * (K + N) * 2
            out[f"nvfp4_{proj}_{name}"] = {"us": round(us, 2), "GB/s": round(nb / us / 1e3, 1),
                                           "frac": round(nb / us / 1e3 / pk["hbm"], 4)}
        del gq, fq
        torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- GPU side: config 2
def run_decode(args) -> None:
    import torch
    import torch.distributed as dist

    from xe2x2_b200 import _lib as L
    from xe2x2_b200 import ops, synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    lib = L.lib()
    fb0 = lib.w4_decode_fallback_count()
    pk = peaks()

    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 2**20) or 126 * 2**20
    wbytes = alg_bytes(0)
    R = max(4, math.ceil(2 * l2 / wbytes) + 1)
    weights = [synth.gptq_weights(K, N, GS, asym=True, seed=1000 * rank + r, device=dev)[:3] for r in range(R)]
    acts = {M: synth.activations(M, K, torch.bfloat16, seed=M, device=dev) for M in MS}
    outs = {M: torch.empty((M, N), dtype=torch.bfloat16, device=dev) for M in MS}
    ws_bytes = max(lib.w4_gptq_workspace_bytes(M, N, K, GS, 0, L.W4_BF16) for M in MS)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)  # the sync area starts zeroed

    def gemm(M, w, out):  # the C-ABI entry point on the current stream
        qw, qz, sc = w
        L.call("w4_gptq_gemm", ops._p(acts[M]), L.W4_BF16, ops._p(qw), ops._p(qz), ops._p(sc), None,
               ops._p(out), L.W4_BF16, None, M, N, K, GS, 1, ops._p(ws), ws_bytes, ops._stream(dev))

    def step():  # ROTATIONS_PER_STEP rotations over the R weight copies of the M-sweep
        for rot in range(ROTATIONS_PER_STEP):
            for r in range(R):
                for j, M in enumerate(MS):
                    gemm(M, weights[(r + j) % R], outs[M])

    gemms_per_step = ROTATIONS_PER_STEP * R * len(MS)
    bytes_per_step = ROTATIONS_PER_STEP * R * sweep_bytes()
    # warm up eagerly (first launches load modules), then capture the step as one graph
    step()
    torch.cuda.synchronize()
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        graph = torch.cuda.CUDAGraph(keep_graph=True)  # kept: its kernel nodes are counted
        with torch.cuda.graph(graph, stream=cap):
            step()
    torch.cuda.current_stream().wait_stream(cap)
    step_kernels = graph_kernels(graph)
    graph.instantiate()
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
    for _ in range(args.warmup):
        graph.replay()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        graph.replay()
    e1.record(st)
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    value = bytes_per_step * args.steps * world / (ms / 1e3) / 1e9

    # ---------------- per-launch kernel durations (roofline of the decode kernel)
    per_m = {}
    for M in MS:
        us = time_graph(lambda r, M=M: gemm(M, weights[r % R], outs[M]), max(30, 2 * R))
        per_m[str(M)] = {"us": round(us, 3), "GB/s": round(alg_bytes(M) / us / 1e3, 1),
                         "frac": round(alg_bytes(M) / us / 1e3 / pk["hbm"], 4)}
    tot_b = sweep_bytes()
    tot_us = sum(per_m[str(M)]["us"] for M in MS)
    achieved = tot_b / tot_us / 1e3

    # ---------------- the read bandwidth one launch of this size attains (w4_read_probe), timed
    # the same way over as many buffers of one M = 1 launch's bytes: the practical ceiling of a
    # GEMM launch that reads its operands once (launch ramp and tail included)
    rb = alg_bytes(1) // 16 * 16
    probe_bufs = [torch.randint(0, 256, (rb,), dtype=torch.uint8, device=dev) for _ in range(R)]
    sink = torch.zeros(1, dtype=torch.int32, device=dev)
    probe_us = time_graph(lambda r: L.call("w4_read_probe", ops._p(probe_bufs[r % R]), rb, ops._p(sink),
                                           ops._stream(dev)), max(30, 2 * R))
    del probe_bufs
    read_ceiling = {"bytes": rb, "us": round(probe_us, 3), "GB/s": round(rb / probe_us / 1e3, 1),
                    "frac_of_peak": round(rb / probe_us / 1e3 / pk["hbm"], 4),
                    "m1_frac_of_ceiling": round(probe_us / per_m["1"]["us"], 4)}

    # ---------------- end to end through the public API (pinned host in, host out)
    # Each step's inputs (the four activation blocks) travel from pinned host memory in one copy
    # and its four outputs come back in one, as a serving loop runs them: copies on their own
    # streams, double-buffered, so step t+1's upload and step t-1's download overlap step t's
    # GEMMs.  G steps (a whole number of weight rotations and of buffer pairs) form one graph.
    rows = sum(MS)
    NB = 2
    h_in = [torch.cat([acts[M].cpu() for M in MS]).pin_memory() for _ in range(NB)]
    h_out = [torch.empty((rows, N), dtype=torch.bfloat16).pin_memory() for _ in range(NB)]
    d_in = [torch.empty((rows, K), dtype=torch.bfloat16, device=dev) for _ in range(NB)]
    d_out = [torch.empty((rows, N), dtype=torch.bfloat16, device=dev) for _ in range(NB)]
    offs = [sum(MS[:j]) for j in range(len(MS))]
    period = R // math.gcd(len(MS), R)
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
    pl = (G - 1) % NB
    g_e2e.replay()
    torch.cuda.synchronize()
    for j, M in enumerate(MS):  # the pipeline's last output against a direct call
        qw, qz, sc = weights[(len(MS) * (G - 1) + j) % R]
        want = ops.gptq_gemm(acts[M], qw, qz, sc, GS, 1)
        if not torch.equal(h_out[pl][offs[j]:offs[j] + M], want.cpu()):
            raise RuntimeError(f"end-to-end pipeline output differs from the direct call at M={M}")
    reps = max(1, -(-args.steps * gemms_per_step // (G * len(MS))))
    for _ in range(max(1, -(-args.warmup // G))):
        g_e2e.replay()
    barrier()
    e0.record(st)
    for _ in range(reps):
        g_e2e.replay()
    e1.record(st)
    barrier()
    e2e_steps_done = reps * G
    ms_e2e = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = sweep_bytes() * e2e_steps_done * world / (ms_e2e / 1e3) / 1e9
    h2d = sum(M * K * 2 for M in MS)
    d2h = sum(M * N * 2 for M in MS)

    fallbacks = lib.w4_decode_fallback_count() - fb0
    graph = None
    del g_e2e
    extra = {}
    if world == 1 and not args.skip_per_config:
        extra["per_config"] = per_config(dev, pk, cpu=not args.no_cpu_baseline)
        extra["tp1"] = tp1_layer_set(dev)
    cpu = cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config_keys(world, R, l2, wbytes, gemms_per_step, bytes_per_step),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "ops.gptq_gemm per M; each M-sweep's activations in one pinned-host copy and its outputs "
                            "out in one, on separate streams with double buffers so copies overlap the neighbouring "
                            f"sweeps' GEMMs; {G}-sweep multi-stream graph replayed",
                    "sweeps": e2e_steps_done, "ms_per_sweep": round(ms_e2e / e2e_steps_done, 5)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm"], "unit": "GB/s",
                         "frac": round(achieved / pk["hbm"], 4), "traffic": TRAFFIC_PER_LAUNCH,
                         "kernel": "w4::dec::gptq_decode_kernel (M = 1, 4, 8), w4::gptq_gemv_kernel (M = 16)",
                         "peak_source": pk["source"] + " hbm_gbs (copy)",
                         "per_m": per_m, "read_ceiling": read_ceiling},
            "gpu_launches": gemms_per_step * args.steps if step_kernels is None else step_kernels["w4"] * args.steps,
            "graph_kernels_per_step": step_kernels,
            "decode_fallbacks": fallbacks,
            "clocks": clk,
        }
        line.update(extra)
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def config_keys(world: int, R: int, l2: int, wbytes: int, gemms_per_step: int, bytes_per_step: int) -> dict:
    """The ``config`` object of the config 2 line (the same keys in both arms)."""
    return {"workload": WORKLOAD,
            "step": f"{ROTATIONS_PER_STEP} rotations over {R} weight copies of the M-sweep "
                    f"({gemms_per_step} GEMMs) replayed from a CUDA graph",
            "l2": f"inputs larger than L2: weights rotate over {R} copies ({R * wbytes / 1e6:.0f} MB vs "
                  f"{l2 / 1e6:.0f} MB L2)",
            "parallelism": f"{world} independent replicas (no data-path collective)" if world > 1 else "single GPU",
            "algorithmic_bytes_per_step": bytes_per_step}


def tp1_layer_set(dev) -> dict:
    """Config 5's layer set on this one GPU (TP=1): the baseline the tensor-parallel runs shard."""
    import torch

    from xe2x2_b200 import tp

    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    sets = [tp.TPLayerSet(None, 0, 1, dev, seed=1000 * r) for r in range(1)]
    R = copies_for(sets[0].weight_bytes_per_rank(), l2)
    sets += [tp.TPLayerSet(None, 0, 1, dev, seed=1000 * r) for r in range(1, R)]
    out = {}
    for M in TP_MS:
        x = sets[0].inputs(M)
        o = {p.name: torch.empty((M, p.N), dtype=torch.bfloat16, device=dev) for p in sets[0].projs}
        us = time_graph(lambda r: sets[r % R].step(x, o), max(R, 6))
        out[str(M)] = {"layer_us": round(us, 2), "TFLOP/s": round(sets[0].flops(M) / us / 1e6, 2),
                       "GB/s": round(sets[0].bytes(M) / us / 1e3, 1)}
    del sets
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- TP layer set (config 5)
TP_MS = (1, 32, 256)
TP_WORKLOAD = ("config5: one 27B-class dense layer's GPTQ g128 projections (QKV N=7168 and gate|up N=34816 "
               "column-parallel, o 5120x5120 and down K=17408 row-parallel with an all-reduce of bf16 "
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
    lib = L.lib()
    fb0 = lib.w4_decode_fallback_count()
    trace("process group up")
    comm = tp.TPComm(rank, world, timeout_ms=120000, device=dev) if world > 1 else None
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

    def step():  # one rotation over the R layer-set copies at every M
        for r in range(R):
            for j, M in enumerate(TP_MS):
                sets[(r + j) % R].step(xs[M], outs[M])

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

    trace(f"{R} layer sets built")
    # eager warm-up on the capture stream: the per-stream workspaces (zero-filled when first
    # allocated) exist before capture, so no fill kernel lands in the step graph
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        step()
    torch.cuda.current_stream().wait_stream(cap)
    if comm is not None:
        comm.wait()
    barrier()
    trace("eager warm-up done")
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        graph = torch.cuda.CUDAGraph(keep_graph=True)  # kept: its kernel nodes are counted
        with torch.cuda.graph(graph, stream=cap):
            step()
    torch.cuda.current_stream().wait_stream(cap)
    step_kernels = graph_kernels(graph)
    graph.instantiate()
    barrier()
    trace(f"graph captured: kernels per step {step_kernels}")
    for _ in range(args.warmup):
        graph.replay()
    if comm is not None:
        comm.wait()
    trace("graph warm-up done")
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        graph.replay()
    e1.record(st)
    trace("timed steps enqueued")
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    trace(f"timed region: {ms:.3f} ms")

    # ---------------- end to end: every step's activations in from pinned host memory, every
    # projection's output back to pinned host memory, around the same rotation (one graph)
    h_xs = {M: {k: v.cpu().pin_memory() for k, v in xs[M].items()} for M in TP_MS}
    h_outs = {M: {k: torch.empty(v.shape, dtype=v.dtype).pin_memory() for k, v in outs[M].items()} for M in TP_MS}

    def e2e_step():
        for M in TP_MS:
            for k in xs[M]:
                xs[M][k].copy_(h_xs[M][k], non_blocking=True)
        step()
        for M in TP_MS:
            for k in outs[M]:
                h_outs[M][k].copy_(outs[M][k], non_blocking=True)

    h2d = sum(t.numel() * t.element_size() for M in TP_MS for t in h_xs[M].values())
    d2h = sum(t.numel() * t.element_size() for M in TP_MS for t in h_outs[M].values())
    with torch.cuda.stream(cap):
        g_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_e2e, stream=cap):
            e2e_step()
    torch.cuda.current_stream().wait_stream(cap)
    for _ in range(args.warmup):
        g_e2e.replay()
    barrier()
    e0.record(st)
    for _ in range(args.steps):
        g_e2e.replay()
    e1.record(st)
    barrier()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1))
    del g_e2e  # holds collective work: gone before the communicator is
    trace(f"e2e region: {ms_e2e:.3f} ms")

    # per-M layer time and all-reduce time alone (graphs of one M / of the bare collectives)
    per_m = {}
    for M in TP_MS:
        gm = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(gm, stream=cap):
                for r in range(R):
                    sets[r].step(xs[M], outs[M])
        torch.cuda.current_stream().wait_stream(cap)
        ga = gu = None
        if comm is not None:
            ga = torch.cuda.CUDAGraph()
            with torch.cuda.stream(cap):
                with torch.cuda.graph(ga, stream=cap):
                    for r in range(R):
                        comm.allreduce_(outs[M]["o"])
                        comm.allreduce_(outs[M]["down"])
            torch.cuda.current_stream().wait_stream(cap)
            if M <= 16:
                # decode sizes: the row-parallel GEMMs reduce in their own epilogue over peer
                # memory (the default is GEMM + one-shot all-reduce)
                comm.set_fused_epilogue(True)
                gu = torch.cuda.CUDAGraph()
                with torch.cuda.stream(cap):
                    with torch.cuda.graph(gu, stream=cap):
                        for r in range(R):
                            sets[r].step(xs[M], outs[M])
                torch.cuda.current_stream().wait_stream(cap)
                comm.set_fused_epilogue(False)
        res = []
        for g in (gm, ga, gu):
            if g is None:
                res.append(0.0)
                continue
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
                         "TFLOP/s": round(sets[0].flops(M) / res[0] / 1e6, 2),
                         "GB/s": round(sets[0].bytes(M) / res[0] / 1e3, 1)}
        if gu is not None:
            per_m[str(M)]["layer_fused_epilogue_us"] = round(res[2], 2)
        del gm, ga, gu  # graphs holding collective work must be gone before the communicator is
    graph = None
    torch.cuda.synchronize()
    if comm is not None:
        comm.close()

    step_bytes_tp = R * sum(sets[0].bytes(M) for M in TP_MS)
    value = step_bytes_tp * args.steps / (ms / 1e3) / 1e9
    e2e_value = step_bytes_tp * args.steps / (ms_e2e / 1e3) / 1e9
    pk = peaks()
    fallbacks = lib.w4_decode_fallback_count() - fb0
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": TP_WORKLOAD, "parallelism": f"tp{world}",
                       "step": f"one rotation over {R} layer-set copies at M=1,32,256 ({12 * R} GEMMs, "
                               f"{6 * R if world > 1 else 0} all-reduces) replayed from a CUDA graph",
                       "l2": f"inputs larger than L2: {R} layer-set copies of {per_rank / 1e6:.1f} MB per rank",
                       "algorithmic_bytes_per_step": step_bytes_tp,
                       "flops_per_step": R * sum(sets[0].flops(M) for M in TP_MS)},
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": round(pk["hbm"] * world, 1),
                         "unit": "GB/s", "frac": round(value / (pk["hbm"] * world), 4), "traffic": None,
                         "peak_source": f"{world} x {pk['source']} hbm_gbs", "per_m": per_m},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "path": "tp.TPLayerSet.step (w4_tp_linear per projection shard); every step copies its "
                            "activations in from pinned host memory and every projection's output back, "
                            "in one CUDA graph per step", "ms_per_step": round(ms_e2e / args.steps, 5)},
            # counted from the step graph; if it cannot be inspected, the lower bound of one libw4
            # kernel per GEMM call (12 per rotation)
            "gpu_launches": (12 * R if step_kernels is None else step_kernels["w4"]) * args.steps,
            "graph_kernels_per_step": step_kernels if step_kernels is not None else "not inspected: lower bound",
            "decode_fallbacks": fallbacks, "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- reference arm
def run_reference(args) -> None:
    """The reference's CPU path (its host loops restated in C: oracle/w4_oracle.c) on a bounded
    sample of the same workload, all host threads, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    O.build()
    cores = os.cpu_count() or 1
    world = args.gpus
    budget = 60.0 / max(1, args.steps + args.warmup)  # the whole run within about a minute
    n_cols = sample_columns(budget, cores)
    weights, acts = cpu_sweep_inputs(0, n_cols)
    for _ in range(args.warmup):
        cpu_sweep(weights, acts, cores)
    times = [cpu_sweep(weights, acts, cores) for _ in range(args.steps)]
    total = sum(times)
    value = sweep_bytes(n_cols) * args.steps / total / 1e9
    l2 = 126 * 2**20
    R = max(4, math.ceil(2 * l2 / alg_bytes(0)) + 1)
    cfg = config_keys(1 if world == 1 else world, R, l2, alg_bytes(0), ROTATIONS_PER_STEP * R * len(MS),
                      ROTATIONS_PER_STEP * R * sweep_bytes())
    cfg["sample_columns"] = n_cols
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": cfg,
        "cpu_baseline": dict({"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                              "sample": f"each step: the M-sweep on {n_cols} of {N} columns; the reference's SYCL host "
                                        "code needs icpx (absent), so its loops run as the plain-C oracle"}, **cpu_info()),
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--skip-per-config", action="store_true", help="only the config 2 headline")
    ap.add_argument("--trace", action="store_true", help="progress lines on stderr")
    ap.add_argument("--workload", choices=["auto", "decode", "tp", "replicas"], default="auto",
                    help="auto: config 2 on one GPU, the config 5 tensor-parallel layer set on several; "
                         "replicas: independent copies of config 2 on every GPU")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "tp" or (args.workload == "auto" and world > 1):
        run_tp(args)
    else:
        run_decode(args)


if __name__ == "__main__":
    main()
