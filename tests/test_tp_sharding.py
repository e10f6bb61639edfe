"""Tensor-parallel sharding on CPU: two gloo ranks, each computing its shard with
the CPU oracle, must reproduce the unsharded layer.

Column shards are concatenated per sub-matrix (q|k|v, gate|up, head-aligned);
row shards are summed with all_reduce, the reference's only TP step
(parallel/tp2/bench_xccl_p2p0.py:235-251: in-place all_reduce(SUM), identity r+1
summed).  The CUDA path (w4_tp_linear + NCCL) is checked by test_tp_gpu.py.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from xe2x2_b200 import synth, tp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _f16_bits(scales):
    return scales.view(torch.int16).numpy().view(np.uint16)


def _qz(qz):
    return None if qz is None else qz.numpy()


def _oracle(a, qw, qz, sc, K, N, gs):
    return O.gptq_gemm(a.float().numpy(), qw.numpy(), _qz(qz), _f16_bits(sc), None, a.shape[0], N, K, gs, 1, threads=1)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gs, M = 64, 3
        # identity check of the reference collective: every rank contributes r+1
        t = torch.full((8,), float(rank + 1))
        dist.all_reduce(t)
        assert torch.all(t == sum(r + 1 for r in range(world)))

        # column-parallel q|k|v with head-aligned sub-matrix splits
        K, splits = 256, (128, 64, 64)
        N = sum(splits)
        qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=3)
        a = synth.activations(M, K, torch.float32, seed=4)
        full = _oracle(a, qw, qz, sc, K, N, gs)
        sqw, sqz, ssc = tp.shard_columns(qw, qz, sc, rank, world, splits)
        part = _oracle(a, sqw, sqz, ssc, K, sqw.shape[1], gs)
        want = np.concatenate([full[:, s] for s in tp.column_slices(splits, rank, world)], axis=1)
        np.testing.assert_array_equal(part, want)

        # row-parallel: K split on group boundaries, partials summed
        K, N = 512, 96
        qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=5)
        a = synth.activations(M, K, torch.float32, seed=6)
        full = _oracle(a, qw, qz, sc, K, N, gs)
        rqw, rqz, rsc = tp.shard_rows(qw, qz, sc, rank, world, gs)
        xs = a[:, tp.row_input_slice(K, rank, world)].contiguous()
        part = torch.from_numpy(_oracle(xs, rqw, rqz, rsc, K // world, N, gs))
        dist.all_reduce(part)
        rel = np.linalg.norm(part.numpy() - full) / np.linalg.norm(full)
        assert rel < 1e-6, rel

        # symmetric (no qzeros) row shard
        rqw, rqz, rsc = tp.shard_rows(qw, None, sc, rank, world, gs)
        assert rqz is None and rqw.shape == (K // world // 8, N)
        q.put((rank, "ok"))
    except Exception as e:  # report, do not hang the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_shards_reproduce_unsharded_layer(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert res == {r: "ok" for r in range(world)}, res


def test_shard_helpers_reject_bad_splits():
    qw, qz, sc, _ = synth.gptq_weights(256, 96, 64, asym=True, seed=0)
    with pytest.raises(ValueError):
        tp.shard_columns(qw, qz, sc, 0, 2, (90, 6))  # does not add up... and not multiples of 8
    with pytest.raises(ValueError):
        tp.shard_columns(qw, qz, sc, 0, 4, (48, 48))  # 12 columns per shard: not a multiple of 8
    with pytest.raises(ValueError):
        tp.shard_rows(qw, qz, sc, 0, 3, 64)  # 256 rows do not split into 3 whole-group shards


def test_dense_layer_shapes_shard_at_tp8():
    for p in tp.dense_27b_projections():
        if p.mode == "column":
            for n in p.splits:
                assert n % 8 == 0 and (n // 8) % 8 == 0 and (n // 8) % 32 == 0
        else:
            assert p.K % (8 * 128) == 0


# ---------------------------------------------------------------- NVFP4 shards
def _fp4_oracle(x, w, scale, gscale):
    K, N = w.shape[0] * 2, w.shape[1]
    return O.nvfp4_gemm(x.float().numpy(), w.contiguous().numpy(), O.NVFP4_KN, scale.view(torch.uint8).numpy(),
                        O.SCALE_E4M3, float(gscale), x.shape[0], N, K, threads=1)


@pytest.mark.parametrize("world", [2, 4])
def test_nvfp4_shards_reproduce_unsharded_layer(world):
    """NVFP4 column shards (q|k|v splits) concatenate to the full product bit for bit; row
    shards (K split on whole 256-k blocks, scale rows following) sum to it within fp32
    rounding; the shards keep the operator layout (stride(0) == 1)."""
    M, K = 3, 1024
    splits = (256, 128, 128)
    N = sum(splits)
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=11)
    x = synth.activations(M, K, torch.bfloat16, seed=12)
    full = _fp4_oracle(x, w, scale, gscale)
    parts = []
    for rank in range(world):
        ws, sc = tp.shard_nvfp4_columns(w, scale, rank, world, splits)
        assert ws.stride(0) == 1 and ws.shape == (K // 2, N // world) and sc.shape == (K // 16, N // world)
        got = _fp4_oracle(x, ws, sc, gscale)
        want = np.concatenate([full[:, s] for s in tp.column_slices(splits, rank, world)], axis=1)
        assert np.array_equal(got, want)
        wr, sr = tp.shard_nvfp4_rows(w, scale, rank, world)
        assert wr.stride(0) == 1 and wr.shape == (K // world // 2, N) and sr.shape == (K // world // 16, N)
        parts.append(_fp4_oracle(x[:, tp.row_input_slice(K, rank, world)].contiguous(), wr, sr, gscale))
    total = np.sum(np.stack(parts), axis=0, dtype=np.float32)
    assert float(np.linalg.norm(total - full) / np.linalg.norm(full)) < 1e-6


def test_nvfp4_shard_helpers_reject_bad_layouts():
    w, scale, _ = synth.nvfp4_weights(512, 128, seed=1)
    with pytest.raises(ValueError, match="stride"):
        tp.shard_nvfp4_columns(w.contiguous(), scale, 0, 2)  # [K/2, N] row-major is not the operator view
    with pytest.raises(ValueError, match="multiple of 256"):
        tp.shard_nvfp4_rows(w, scale, 0, 4)  # 512 / 4 = 128 k per shard
    with pytest.raises(ValueError):
        tp.TPLinearNVFP4(None, "row", w, scale, torch.ones(1))
