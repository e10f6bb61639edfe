"""Tensor-parallel layers on 2 GPUs: w4_tp_linear (column / row) through libw4's
NCCL communicator against the unsharded single-GPU GEMM, the collective's
identity check (parallel/tp2/bench_xccl_p2p0.py:235-245: ranks add r+1), and
the bounded waits: a rank that never joins the communicator, or never reaches
a collective, makes the other rank's call return W4_ERR_TIMEOUT.  The NVFP4
layers (TPLinearNVFP4, bf16 and NVFP4 activations) against the unsharded
NVFP4 GEMM.

Each case runs as child processes (one per GPU) bootstrapped over gloo, with
NVLS off (NCCL_NVLS_ENABLE=0).  A rank leaves only between steps, with
nothing of its own in flight.  The layer cases run at 2 ranks and at
min(4, GPU count) ranks; everything is skipped with fewer than 2 GPUs.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rel(x, y):
    x, y = x.float(), y.float()
    return float((x - y).norm() / y.norm())


def _case_layers(rank, world):
    from xe2x2_b200 import _lib as L, ops, synth, tp

    dev = torch.device("cuda", rank)
    comm = tp.TPComm(rank, world, timeout_ms=60000, device=dev)
    try:
        # identity check of the collective (one-shot peer-memory path for small messages,
        # NCCL above its slot size)
        for n in (4096, 8, 40000, 1 << 20):
            t = torch.full((n,), float(rank + 1), dtype=torch.bfloat16, device=dev)
            comm.allreduce_(t)
            comm.wait()
            assert torch.all(t == float(sum(r + 1 for r in range(world)))), n
        # every rank ends with the same bits, in f32 too
        g = torch.Generator(device=dev).manual_seed(rank)
        x = torch.randn(12288, generator=g, device=dev)
        ref = sum(torch.randn(12288, generator=torch.Generator(device=dev).manual_seed(r), device=dev)
                  for r in range(world))
        comm.allreduce_(x)
        comm.wait()
        assert torch.allclose(x, ref, rtol=1e-6, atol=1e-6)
        # captured in a CUDA graph and replayed: the per-call counters live on the device
        y = torch.zeros(5120, dtype=torch.bfloat16, device=dev)
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            y.fill_(float(rank + 1))
            comm.allreduce_(y)  # warm-up outside capture
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(graph, stream=st):
                y.fill_(float(rank + 1))
                comm.allreduce_(y)
                y.mul_(2.0)
                comm.allreduce_(y)
        torch.cuda.current_stream(dev).wait_stream(st)
        for _ in range(3):
            graph.replay()
            comm.wait()
            assert torch.all(y == float(2 * world * sum(r + 1 for r in range(world))))
        del graph

        gs = 128
        for M in (1, 32, 256):
            # column-parallel QKV-like matrix with head-aligned splits
            K, splits = 1024, (512, 256, 256)
            N = sum(splits)
            qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=11, device=dev)
            a = synth.activations(M, K, torch.bfloat16, seed=M, device=dev)
            full = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float32)
            lay = tp.TPLinear(comm, "column", *tp.shard_columns(qw, qz, sc, rank, world, splits), group_size=gs)
            got = lay(a, out_dtype=torch.float32)
            want = torch.cat([full[:, s] for s in tp.column_slices(splits, rank, world)], dim=1)
            assert _rel(got, want) < 1e-6

            # row-parallel: f32, bf16 and fp8 row-scaled outputs
            K, N = 2048, 512
            qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=12, device=dev)
            a = synth.activations(M, K, torch.bfloat16, seed=100 + M, device=dev)
            full = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float32)
            lay = tp.TPLinear(comm, "row", *tp.shard_rows(qw, qz, sc, rank, world, gs), group_size=gs)
            xs = a[:, tp.row_input_slice(K, rank, world)].contiguous()
            got32 = lay(xs, out_dtype=torch.float32)
            got16 = lay(xs, out_dtype=torch.bfloat16)
            q8, rs = lay(xs, out_dtype=torch.float8_e4m3fn)
            comm.wait()
            assert _rel(got32, full) < 1e-5
            assert _rel(got16, full) < 1e-2
            deq = q8.float() * rs[:, None]
            assert _rel(deq, full) < 4e-2
            ref_rs = full.abs().amax(dim=1) / 448.0
            assert torch.allclose(rs, ref_rs, rtol=1e-5)
        assert L.lib().w4_check_device_status() == L.W4_OK
    finally:
        comm.close()


def _case_fused_row_parallel(rank, world):
    """Decode row-parallel layers reducing in the GEMV epilogue over peer memory
    (w4_tp_set_fused_epilogue): equal to GEMM + all-reduce up to fp32 summation order, the same bits on every rank,
    correct under CUDA-graph replay, close to the unsharded GEMM."""
    import torch.distributed as dist

    from xe2x2_b200 import _lib as L, ops, synth, tp

    dev = torch.device("cuda", rank)
    comm = tp.TPComm(rank, world, timeout_ms=60000, device=dev)
    try:
        gs = 128
        for K, N in ((2048, 5120), (4096, 1024)):
            qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=K + N, device=dev)
            lay = tp.TPLinear(comm, "row", *tp.shard_rows(qw, qz, sc, rank, world, gs), group_size=gs)
            for M in (1, 4, 9, 16):
                a = synth.activations(M, K, torch.bfloat16, seed=M, device=dev)
                xs = a[:, tp.row_input_slice(K, rank, world)].contiguous()
                full = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float32)
                comm.set_fused_epilogue(True)
                f32 = lay(xs, out_dtype=torch.float32)
                b16 = lay(xs, out_dtype=torch.bfloat16)
                q8, rs = lay(xs, out_dtype=torch.float8_e4m3fn)
                comm.set_fused_epilogue(False)
                u32 = lay(xs, out_dtype=torch.float32)
                comm.wait()
                # exact products either way; the fused and the un-fused GEMMs sum them in fp32 in
                # different orders (the un-fused one per 128-k unit and over a K split), each with
                # codes entering the MMA as 1024 + q: an fp32 sum about 128x the result's size,
                # hence up to ~1e-5 from the exact product each (the contract allows 1e-2)
                assert _rel(f32, u32) < 5e-5, (K, N, M)
                assert _rel(f32, full) < 5e-5
                assert _rel(b16, full) < 1e-2
                assert _rel(q8.float() * rs[:, None], full) < 4e-2
                got = [torch.empty_like(f32.cpu()) for _ in range(world)]
                dist.all_gather(got, f32.cpu())
                assert all(torch.equal(g, got[0]) for g in got)
        # CUDA-graph replay: the call sequence lives on the device
        comm.set_fused_epilogue(True)
        K, N, M = 2048, 5120, 2
        qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=77, device=dev)
        lay = tp.TPLinear(comm, "row", *tp.shard_rows(qw, qz, sc, rank, world, gs), group_size=gs)
        a = synth.activations(M, K, torch.bfloat16, seed=78, device=dev)
        xs = a[:, tp.row_input_slice(K, rank, world)].contiguous()
        want = lay(xs, out_dtype=torch.float32)
        comm.wait()
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            lay(xs, out_dtype=torch.float32)
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(graph, stream=st):
                y1 = lay(xs, out_dtype=torch.float32)
                y2 = lay(xs, out_dtype=torch.float32)
        torch.cuda.current_stream(dev).wait_stream(st)
        for _ in range(3):
            graph.replay()
            comm.wait()
            assert torch.equal(y1, want) and torch.equal(y2, want)
        del graph
        assert L.lib().w4_check_device_status() == L.W4_OK
    finally:
        comm.close()


def _case_fused_timeout(rank, world):
    """Rank 1 skips one fused row-parallel call (it launches nothing): rank 0's CTAs
    stop waiting after their time limit and the wait reports W4_ERR_TIMEOUT."""
    import torch.distributed as dist

    from xe2x2_b200 import _lib as L, synth, tp

    dev = torch.device("cuda", rank)
    comm = tp.TPComm(rank, world, timeout_ms=60000, device=dev)
    comm.set_fused_epilogue(True)
    K, N, gs = 1024, 512, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=5, device=dev)
    lay = tp.TPLinear(comm, "row", *tp.shard_rows(qw, qz, sc, rank, world, gs), group_size=gs)
    xs = synth.activations(1, K // world, torch.bfloat16, seed=6, device=dev)
    lay(xs)
    comm.wait()
    dist.barrier()  # every rank is between steps
    if rank == 0:
        lay(xs)
        with pytest.raises(L.W4Error) as ei:
            comm.wait(timeout_ms=20000)
        assert ei.value.status == L.W4_ERR_TIMEOUT
        torch.cuda.synchronize(dev)  # the kernel gave up and left the GPU
    dist.barrier()
    comm.abort()


def _case_init_timeout(rank, world):
    """Rank 1 never joins: rank 0's communicator init gives up with W4_ERR_TIMEOUT."""
    import ctypes

    import torch.distributed as dist

    from xe2x2_b200 import _lib as L

    buf = (ctypes.c_uint8 * L.W4_TP_UNIQUE_ID_BYTES)()
    if rank == 0:
        L.call("w4_tp_get_unique_id", ctypes.cast(buf, ctypes.c_void_p))
    dist.barrier()
    if rank == 0:
        torch.cuda.set_device(0)
        h = ctypes.c_void_p()
        rc = L.lib().w4_tp_comm_init(ctypes.byref(h), world, 0, ctypes.cast(buf, ctypes.c_void_p), 2000)
        assert rc == L.W4_ERR_TIMEOUT, (rc, L.lib().w4_last_error())
        assert not h.value
    dist.barrier()


def _case_collective_timeout(rank, world):
    """Rank 1 skips one all-reduce (it enqueues nothing): rank 0's bounded wait
    aborts its communicator and reports W4_ERR_TIMEOUT; both ranks then tear
    down without waiting for each other."""
    import torch.distributed as dist

    from xe2x2_b200 import _lib as L, tp

    dev = torch.device("cuda", rank)
    comm = tp.TPComm(rank, world, timeout_ms=60000, device=dev)
    t = torch.ones(1024, dtype=torch.float32, device=dev)
    comm.allreduce_(t)
    comm.wait()
    assert torch.all(t == world)
    dist.barrier()  # every rank is between steps
    if rank == 0:
        comm.allreduce_(t)
        with pytest.raises(L.W4Error) as ei:
            comm.wait(timeout_ms=1500)
        assert ei.value.status == L.W4_ERR_TIMEOUT
        comm.abort()
        torch.cuda.synchronize(dev)  # the aborted collective has left the GPU
    dist.barrier()
    if rank != 0:
        comm.abort()


def _case_nvfp4_layers(rank, world):
    """TPLinearNVFP4 column and row shards (bf16 activations, and NVFP4 activations with the
    layer's tensor scale) against the unsharded NVFP4 GEMM on the same inputs."""
    from xe2x2_b200 import _lib as L, ops, synth, tp

    dev = torch.device("cuda", rank)
    comm = tp.TPComm(rank, world, timeout_ms=60000, device=dev)
    try:
        K, N = 2048, 1536
        splits = (1024, 256, 256)
        w, scale, gscale = synth.nvfp4_weights(K, N, seed=21, device=dev)
        for M in (1, 16, 256):
            x = synth.activations(M, K, torch.bfloat16, seed=M, device=dev)
            ag = torch.tensor([float(x.float().abs().max()) / (448.0 * 6.0)], device=dev)
            for act_mode, a_global, tol in ((L.W4_ACT_W4A16, None, 1e-5), (L.W4_ACT_NVFP4, ag, 1e-5)):
                full = ops.nvfp4_gemm(x, w, scale, gscale, torch.float32, act_mode, a_global)
                ws, sc = tp.shard_nvfp4_columns(w, scale, rank, world, splits)
                col = tp.TPLinearNVFP4(comm, "column", ws, sc, gscale, act_mode, a_global)
                got = col(x, out_dtype=torch.float32)
                want = torch.cat([full[:, s] for s in tp.column_slices(splits, rank, world)], dim=1)
                assert _rel(got, want) < tol, (M, act_mode)
                wr, sr = tp.shard_nvfp4_rows(w, scale, rank, world)
                row = tp.TPLinearNVFP4(comm, "row", wr, sr, gscale, act_mode, a_global)
                xs = x[:, tp.row_input_slice(K, rank, world)].contiguous()
                got = row(xs, out_dtype=torch.float32)
                b16 = row(xs, out_dtype=torch.bfloat16)
                comm.wait()
                # NVFP4 activations: the shard quantises its own K slice with the same global scale
                # and 16-element blocks, so the codes match the unsharded quantiser's
                assert _rel(got, full) < 1e-5, (M, act_mode)
                assert _rel(b16, full) < 1e-2, (M, act_mode)
        assert L.lib().w4_check_device_status() == L.W4_OK
    finally:
        comm.close()


def _child(rank, world, port, case, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        globals()[case](rank, world)
        q.put((rank, "ok"))
    except BaseException as e:  # report to the parent rather than hang it
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _run(case, world=WORLD):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_child, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=300)
            res[r] = v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res == {r: "ok" for r in range(world)}, res


def _worlds():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return sorted({2, max(2, min(4, n))})


@pytest.mark.parametrize("world", _worlds())
def test_tp_layers_match_unsharded(world):
    _run("_case_layers", world)


@pytest.mark.parametrize("world", _worlds())
def test_tp_fused_row_parallel_epilogue(world):
    _run("_case_fused_row_parallel", world)


@pytest.mark.parametrize("world", _worlds())
def test_tp_nvfp4_layers_match_unsharded(world):
    _run("_case_nvfp4_layers", world)


def test_tp_fused_epilogue_timeout_when_a_rank_skips():
    _run("_case_fused_timeout")


def test_tp_init_timeout_when_a_rank_never_joins():
    _run("_case_init_timeout")


def test_tp_collective_timeout_when_a_rank_skips():
    _run("_case_collective_timeout")
