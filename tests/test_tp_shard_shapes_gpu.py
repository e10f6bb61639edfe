"""Oracle parity of every rank's shard of BASELINE config 5 (one 27B-class dense layer's
GPTQ projections) at TP = 2, 4 and 8, on one GPU.

Each shard is an ordinary GEMM on the rank that holds it: QKV and gate|up split by
columns (head-aligned: 5120/TP query columns and 1024/TP of each of K and V), o and down
split by rows.  The row shards at TP=8 have odd group counts (o: K=640 = 5 groups of 128;
down: K=2176 = 17 groups), which the decode and prefill GEMMs must handle whole.  The
shard is cut by the same helpers the tensor-parallel layers use (xe2x2_b200/tp.py) and
compared with the host oracle on the shard's own inputs.
"""
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, bits16, f32, np_
from xe2x2_b200 import ops, synth, tp

pytestmark = pytest.mark.gpu

GS = 128
PROJS = {p.name: p for p in tp.dense_27b_projections()}
SEEDS = {"qkv": 1, "o": 2, "gate_up": 3, "down": 4}


def _shard(p, rank, world, device):
    # one seeded full matrix per projection, cut like TPLayerSet does
    qw, qz, sc, _ = synth.gptq_weights(p.K, p.N, GS, asym=True, seed=SEEDS[p.name], device=device)
    if p.mode == "column":
        return tp.shard_columns(qw, qz, sc, rank, world, p.splits)
    return tp.shard_rows(qw, qz, sc, rank, world, GS)


@pytest.mark.parametrize("M", [1, 16, 32])
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("name", ["qkv", "o", "gate_up", "down"])
def test_shard_matches_oracle(cuda, name, world, M):
    p = PROJS[name]
    for rank in sorted({0, world - 1}):
        qw, qz, sc = (t.contiguous() for t in _shard(p, rank, world, cuda))
        K, N = qw.shape[0] * 8, qw.shape[1]
        if p.mode == "row":
            assert K == p.K // world and N == p.N
        else:
            assert K == p.K and N == p.N // world
        a = synth.activations(M, K, torch.bfloat16, seed=M + 31 * rank, device=cuda)
        out = ops.gptq_gemm(a, qw, qz, sc, GS, 1)
        ref = O.gptq_gemm(f32(a), np_(qw), np_(qz), bits16(sc), None, M, N, K, GS, 1)
        assert_gemm_close(f32(out), ref)
        if M <= 16:
            # fp32 output of the decode GEMM: exact products, so only the fp32 summation order
            # separates it from the oracle (from 17 tokens the tensor-core GEMM rounds the
            # dequantized weights to the activation type)
            out32 = ops.gptq_gemm(a, qw, qz, sc, GS, 1, out_dtype=torch.float32)
            assert_gemm_close(np_(out32), ref, rel=1e-4, nmax=1e-4)


@pytest.mark.parametrize("K", [640, 2176, 128, 384])
@pytest.mark.parametrize("M", [1, 5, 16])
def test_odd_group_counts(cuda, K, M):
    """K of an odd number of 128-groups (and a single group) through the decode GEMM."""
    N = 1024
    qw, qz, sc, _ = synth.gptq_weights(K, N, GS, asym=True, seed=K + M, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=K, device=cuda)
    out = ops.gptq_gemm(a, qw, qz, sc, GS, 1, out_dtype=torch.float32)
    ref = O.gptq_gemm(f32(a), np_(qw), np_(qz), bits16(sc), None, M, N, K, GS, 1)
    assert_gemm_close(np_(out), ref, rel=1e-4, nmax=1e-4)
