"""Launch or time one libw4 GEMM shape (for ncu captures and quick per-shape timings).

    python -m xe2x2_b200.profile_driver --kernel gptq --M 16 --K 5120 --N 17408 --iters 4
    python -m xe2x2_b200.profile_driver --kernel nvfp4 --M 1,16 --K 5120 --N 5120 --time
    python -m xe2x2_b200.profile_driver --kernel gptq_grouped --counts 1,1,0,1,1,1,0,1 --K 2688 --N 1856

Without --time it runs ``--iters`` launches back to back (a small, fixed number of
launches for an ncu capture).  With --time it reports the median per-launch
CUDA-event time and the algorithmic GB/s (weights rotate over enough copies to
exceed twice the L2, so each launch reads its weights from HBM).
"""
from __future__ import annotations

import argparse
import json
import math
import statistics

import torch

from . import _lib as L
from . import ops, synth


def time_launches(fn, reps: int) -> list[float]:
    """Per-launch device time (us) of ``fn(i)`` for i in range(reps).

    A GPU sleep kernel is queued first so every launch and event is already
    enqueued when the GPU reaches them: host launch overhead is excluded and the
    events measure back-to-back device time.
    """
    st = torch.cuda.current_stream()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    torch.cuda._sleep(int(reps * 80e-6 * 2.0e9))
    evs[0].record(st)
    for r in range(reps):
        fn(r)
        evs[r + 1].record(st)
    torch.cuda.synchronize()
    return [evs[i].elapsed_time(evs[i + 1]) * 1e3 for i in range(reps)]


def time_graph(fn, reps: int) -> float:
    """Mean device time (us) of one ``fn(i)`` with ``reps`` calls captured in one
    CUDA graph and replayed (no host work between launches)."""
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
    return e0.elapsed_time(e1) * 1e3 / (5 * reps)


def gptq_bytes(M, K, N, gs, asym=True):
    return K // 8 * N * 4 + K // gs * N * 2 + (K // gs * N // 8 * 4 if asym else 0) + M * K * 2 + M * N * 2


def nvfp4_bytes(M, K, N):
    return N * K // 2 + K // 16 * N + 4 + M * K * 2 + M * N * 2


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", choices=["gptq", "nvfp4", "producer", "gptq_grouped", "nvfp4_grouped"],
                    default="gptq", help="producer: the fused RMSNorm -> NVFP4 activation kernel on [M, K]; "
                    "*_grouped: one grouped (MoE) launch over len(--counts) experts")
    ap.add_argument("--counts", default="1,1,0,1,1,1,0,1", help="tokens per expert of a grouped launch")
    ap.add_argument("--M", default="16", help="comma-separated token counts")
    ap.add_argument("--K", type=int, default=5120)
    ap.add_argument("--N", type=int, default=17408)
    ap.add_argument("--gs", type=int, default=128)
    ap.add_argument("--dtype", choices=["bf16", "f16"], default="bf16")
    ap.add_argument("--iters", type=int, default=4)
    ap.add_argument("--time", action="store_true")
    ap.add_argument("--act", choices=["w4a16", "nvfp4"], default="w4a16",
                    help="NVFP4 kernel: bf16 activations (w4a16) or activations quantised to NVFP4")
    args = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    K, N = args.K, args.N
    wbytes = gptq_bytes(0, K, N, args.gs) if args.kernel == "gptq" else nvfp4_bytes(0, K, N)
    if args.kernel.endswith("_grouped"):
        return grouped(args, dev, dt)
    if args.kernel == "producer":
        wbytes = 1 << 40  # no weights: one copy
    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 << 20) or (126 << 20)
    copies = max(1, math.ceil(2 * l2 / wbytes) + 1) if args.time else 1
    if args.kernel == "gptq":
        ws = [synth.gptq_weights(K, N, args.gs, asym=True, seed=s, device=dev)[:3] for s in range(copies)]
    elif args.kernel == "producer":
        copies = 1  # no weights; inputs are the activations
        ws = [None]
    else:
        ws = [synth.nvfp4_weights(K, N, seed=s, device=dev) for s in range(copies)]
    results = []
    for M in [int(m) for m in args.M.split(",")]:
        a = synth.activations(M, K, dt, seed=M, device=dev)
        ag = torch.tensor([float(a.float().abs().max()) / (448.0 * 6.0)], dtype=torch.float32, device=dev)
        act_mode = L.W4_ACT_NVFP4 if args.act == "nvfp4" else L.W4_ACT_W4A16

        def run(i):
            w = ws[i % copies]
            if args.kernel == "gptq":
                return ops.gptq_gemm(a, w[0], w[1], w[2], args.gs, 1)
            if args.kernel == "producer":
                return ops.rmsnorm_quant_nvfp4(a, ag)
            return ops.nvfp4_gemm(a, w[0], w[1], w[2], act_mode=act_mode, a_global=ag)

        if not args.time:
            for i in range(args.iters):
                run(i)
            torch.cuda.synchronize()
            continue
        for i in range(max(3, copies)):
            run(i)
        us = statistics.median(time_launches(run, max(args.iters, 20)))
        gus = time_graph(run, max(args.iters, 20, copies))
        nb = gptq_bytes(M, K, N, args.gs) if args.kernel == "gptq" else nvfp4_bytes(M, K, N)
        if args.kernel == "producer":
            nb = 2 * M * K + M * K // 2 + M * K // 16
        results.append({"kernel": args.kernel, "M": M, "K": K, "N": N, "us": round(us, 3), "graph_us": round(gus, 3),
                        "GB/s": round(nb / us / 1e3, 1), "TFLOP/s": round(2 * M * N * K / us / 1e6, 2)})
    for r in results:
        print(json.dumps(r))
    print("ok")


def grouped(args, dev, dt):
    """Grouped (MoE) launches: experts of K x N with --counts tokens each, stacked weights."""
    K, N = args.K, args.N
    cnt = [int(c) for c in args.counts.split(",")]
    E = len(cnt)
    off = [0]
    for c in cnt:
        off.append(off[-1] + c)
    a = synth.activations(off[-1], K, dt if args.kernel == "gptq_grouped" else torch.bfloat16, seed=1, device=dev)
    if args.kernel == "gptq_grouped":
        ws = [synth.gptq_weights(K, N, args.gs, asym=True, seed=e, device=dev)[:3] for e in range(E)]
        qw, qz, sc = (torch.stack([w[i] for w in ws]).contiguous() for i in range(3))

        def run(i):
            return ops.gptq_gemm_grouped(a, qw, qz, sc, off, args.gs, 1)
        nb = sum(1 for c in cnt if c) * gptq_bytes(0, K, N, args.gs)
    else:
        ws = [synth.nvfp4_weights(K, N, seed=e, device=dev) for e in range(E)]
        w_nk = torch.stack([w[0].t() for w in ws]).contiguous()
        scale = torch.stack([w[1] for w in ws]).contiguous()
        gsc = torch.cat([w[2] for w in ws]).contiguous()

        def run(i):
            return ops.nvfp4_gemm_grouped(a, w_nk, scale, gsc, off)
        nb = sum(1 for c in cnt if c) * nvfp4_bytes(0, K, N)
    for i in range(args.iters):
        run(i)
    torch.cuda.synchronize()
    if args.time:
        us = time_graph(run, max(args.iters, 20))
        print(json.dumps({"kernel": args.kernel, "counts": cnt, "K": K, "N": N, "graph_us": round(us, 3),
                          "GB/s": round(nb / us / 1e3, 1), "note": "weights of one stack (L2-warm if small)"}))
    print("ok")


if __name__ == "__main__":
    main()
