"""Grouped (MoE) GEMMs: one launch over a list of experts with ragged token counts, against the
host oracle per expert (the reference chains the routed experts of a layer as separate GEMMs,
kernels/esimd_dpas/moe_group_s8_m1.cpp:1-7; expert shapes hidden 2688 x expert 1856,
kernels/nemotron/README.md)."""
import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, bits16, f32, np_
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu

HIDDEN, EXPERT = 2688, 1856
COUNTS = {
    "decode": [3, 0, 1, 7, 2, 16, 5, 1],      # one token block per expert, one expert empty
    "ragged": [20, 1, 0, 33, 9, 2, 17, 4],    # experts past 16 rows: the tensor-core grouped GEMM
    "batch": [24, 31, 0, 17, 40, 29, 33, 18],  # 32 tokens x top 6 over 8 experts
    "heavy": [150, 3, 0, 200, 17, 1, 0, 9],   # experts past 128 rows: two A tiles per CTA
    "one": [0, 0, 20, 0, 0, 0, 0, 0],         # one expert, few tiles: split K
}
# The tensor-core GEMM (an expert with more than 16 rows) rounds each dequantised GPTQ weight
# to bf16 once; the decode kernels and the NVFP4 dequantisation are exact.
GPTQ_BF16_REL = 4e-3


def _tensor_core(cnt):
    return max(cnt) > 16


def _offsets(counts):
    return [0] + list(np.cumsum(counts))


def _gptq_stack(E, K, N, gs, seed):
    ws = [synth.gptq_weights(K, N, gs, asym=True, seed=seed + e, device="cuda")[:3] for e in range(E)]
    return tuple(torch.stack([w[i] for w in ws]).contiguous() for i in range(3))


@pytest.mark.parametrize("counts", list(COUNTS))
@pytest.mark.parametrize("proj,K,N,gs", [("up", HIDDEN, EXPERT, 128), ("down", EXPERT, HIDDEN, 64)])
def test_gptq_grouped_matches_oracle(cuda, counts, proj, K, N, gs):
    cnt = COUNTS[counts]
    E, off = len(cnt), _offsets(cnt)
    qw, qz, sc = _gptq_stack(E, K, N, gs, seed=K)
    a = synth.activations(off[-1], K, torch.bfloat16, seed=3, device=cuda)
    out = ops.gptq_gemm_grouped(a, qw, qz, sc, off, gs, 1)
    out32 = ops.gptq_gemm_grouped(a, qw, qz, sc, off, gs, 1, out_dtype=torch.float32)
    for e in range(E):
        r0, r1 = off[e], off[e + 1]
        if r0 == r1:
            continue
        ref = O.gptq_gemm(f32(a[r0:r1]), np_(qw[e]), np_(qz[e]), bits16(sc[e]), None, r1 - r0, N, K, gs, 1)
        assert_gemm_close(f32(out[r0:r1]), ref)
        if _tensor_core(cnt):
            rf, _ = assert_gemm_close(np_(out32[r0:r1]), ref)
            assert rf < GPTQ_BF16_REL, (e, rf)
        else:
            assert_gemm_close(np_(out32[r0:r1]), ref, rel=1e-4, nmax=1e-4)
    from xe2x2_b200 import _lib as L
    assert L.lib().w4_check_device_status() == L.W4_OK


@pytest.mark.parametrize("counts", ["decode", "batch"])
def test_gptq_grouped_equals_per_expert_calls_and_fp8(cuda, counts):
    """The grouped launch gives each expert what a plain call on its slice gives (to fp32
    summation order: a plain call may run another kernel or K split, with another order of the
    fp32 sums), and the fp8 output is the row-scaled cast of the f32 product."""
    cnt = COUNTS[counts]
    E, off = len(cnt), _offsets(cnt)
    K, N, gs = HIDDEN, EXPERT, 128
    qw, qz, sc = _gptq_stack(E, K, N, gs, seed=5)
    a = synth.activations(off[-1], K, torch.bfloat16, seed=4, device=cuda)
    y = ops.gptq_gemm_grouped(a, qw, qz, sc, off, gs, 1, out_dtype=torch.float32)
    for e in range(E):
        if off[e] == off[e + 1]:
            continue
        one = ops.gptq_gemm(a[off[e]:off[e + 1]].contiguous(), qw[e], qz[e], sc[e], gs, 1, out_dtype=torch.float32)
        rel = float((one - y[off[e]:off[e + 1]]).norm() / one.norm())
        assert rel < 5e-5, (e, rel)
    q, s = ops.gptq_gemm_grouped(a, qw, qz, sc, off, gs, 1, out_dtype=torch.float8_e4m3fn)
    q_ref, s_ref = O.rowscale_fp8(np_(y))
    assert np.array_equal(np_(q.view(torch.uint8)), q_ref)
    assert np.array_equal(np_(s), s_ref)


def _nvfp4_stack(E, K, N, seed):
    ws = [synth.nvfp4_weights(K, N, seed=seed + e, device="cuda") for e in range(E)]
    w_nk = torch.stack([w[0].t() for w in ws]).contiguous()  # [E, N, K/2]
    scale = torch.stack([w[1] for w in ws]).contiguous()      # [E, K/16, N] e4m3
    gsc = torch.cat([w[2] for w in ws]).contiguous()           # [E]
    return w_nk, scale, gsc


@pytest.mark.parametrize("counts", list(COUNTS))
@pytest.mark.parametrize("proj,K,N", [("up", HIDDEN, EXPERT), ("down", EXPERT, HIDDEN)])
def test_nvfp4_grouped_matches_oracle(cuda, counts, proj, K, N):
    cnt = COUNTS[counts]
    E, off = len(cnt), _offsets(cnt)
    w_nk, scale, gsc = _nvfp4_stack(E, K, N, seed=K)
    x = synth.activations(off[-1], K, torch.bfloat16, seed=6, device=cuda)
    out = ops.nvfp4_gemm_grouped(x, w_nk, scale, gsc, off)
    out32 = ops.nvfp4_gemm_grouped(x, w_nk, scale, gsc, off, torch.float32)
    for e in range(E):
        r0, r1 = off[e], off[e + 1]
        if r0 == r1:
            continue
        ref = O.nvfp4_gemm(f32(x[r0:r1]), np_(w_nk[e]), O.NVFP4_NK, np_(scale[e].view(torch.uint8)), 0,
                           float(gsc[e]), r1 - r0, N, K)
        assert_gemm_close(f32(out[r0:r1]), ref)
        assert_gemm_close(np_(out32[r0:r1]), ref, rel=1e-4, nmax=1e-4)
    from xe2x2_b200 import _lib as L
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_nvfp4_grouped_batch_equals_per_expert_calls(cuda):
    """At batch sizes each expert's rows equal a plain W4A16 call on its slice (both on the
    tensor cores; only the fp32 order of a K split may differ)."""
    cnt = COUNTS["batch"]
    E, off = len(cnt), _offsets(cnt)
    K, N = HIDDEN, EXPERT
    w_nk, scale, gsc = _nvfp4_stack(E, K, N, seed=9)
    x = synth.activations(off[-1], K, torch.bfloat16, seed=2, device=cuda)
    y = ops.nvfp4_gemm_grouped(x, w_nk, scale, gsc, off, torch.float32)
    for e in range(E):
        if off[e] == off[e + 1]:
            continue
        w_kn = w_nk[e].t().contiguous()
        one = ops.nvfp4_gemm(x[off[e]:off[e + 1]].contiguous(), w_kn, scale[e], gsc[e:e + 1], out_dtype=torch.float32)
        rel = float((one - y[off[e]:off[e + 1]]).norm() / one.norm())
        assert rel < 5e-6, (e, rel)


def test_grouped_rejects_bad_offsets(cuda):
    from xe2x2_b200 import _lib as L
    qw, qz, sc = _gptq_stack(2, 256, 64, 128, seed=1)
    a = synth.activations(4, 256, torch.bfloat16, seed=1, device=cuda)
    with pytest.raises(L.W4Error):
        ops.gptq_gemm_grouped(a, qw, qz, sc, [1, 2, 4], 128, 1)   # offsets[0] != 0
    with pytest.raises(L.W4Error):
        ops.gptq_gemm_grouped(a[:2].contiguous(), qw, qz, sc, [0, 3, 2], 128, 1)   # decreasing
