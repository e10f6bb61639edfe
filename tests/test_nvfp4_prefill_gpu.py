"""NVFP4 x NVFP4 block-scaled GEMM (tcgen05 kind::mxf4nvf4, act_mode W4_ACT_NVFP4)
vs the CPU oracle: activations quantised by the oracle's NVFP4 quantiser
(bit-exact with w4_nvfp4_quant_act), dequantised, and multiplied in fp32 with
the dequantised weights.  The operands the tensor core sees are therefore the
same values as the oracle's, and only the fp32 summation order differs.
"""
import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, f32, np_
from xe2x2_b200 import _lib as L
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu


def _a_global(x):
    return torch.tensor([float(x.float().abs().max()) / (448.0 * 6.0)], dtype=torch.float32, device=x.device)


def _oracle(x, w, scale, gscale, a_global, rows=None):
    """fp32 product of the NVFP4-quantised activations (rows subset) with the NVFP4 weights."""
    xs = x if rows is None else x[rows]
    M, K = xs.shape
    N = w.shape[1]
    codes, sf = O.nvfp4_quant_act(f32(xs), float(a_global.item()))
    a_deq = O.nvfp4_act_dequant(codes, sf, float(a_global.item()), M, K)
    sc = np_(scale.view(torch.uint8))
    return O.nvfp4_gemm(a_deq, np_(w.contiguous()), O.NVFP4_KN, sc, O.SCALE_E4M3, float(gscale.item()), M, N, K)


@pytest.mark.parametrize("M,K,N,out", [
    (128, 1024, 256, torch.float32),
    (200, 2048, 384, torch.bfloat16),   # M tail
    (1, 512, 128, torch.float32),       # one token, padded tile
    (300, 5120, 640, torch.float16),
])
def test_nvfp4_act_gemm_shapes(cuda, M, K, N, out):
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=M + K, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=M, device=cuda)
    ag = _a_global(x)
    got = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=out, act_mode=L.W4_ACT_NVFP4, a_global=ag)
    assert got.dtype == out and got.shape == (M, N)
    ref = _oracle(x, w, scale, gscale, ag)
    rf, _ = assert_gemm_close(f32(got), ref)
    if out == torch.float32:
        assert rf < 1e-5, rf  # identical operands, fp32 sums
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_nvfp4_act_gemm_fp8_rowscale(cuda):
    M, K, N = 130, 1024, 256
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=5, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=6, device=cuda)
    ag = _a_global(x)
    q8, rs = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float8_e4m3fn, act_mode=L.W4_ACT_NVFP4,
                            a_global=ag)
    ref = _oracle(x, w, scale, gscale, ag)
    assert np.allclose(np_(rs), np.abs(ref).max(axis=1) / 448.0, rtol=1e-4)
    assert_gemm_close(np_(q8.float() * rs[:, None]), ref, rel=4e-2, nmax=8e-2)


def test_nvfp4_act_rejects_unsupported(cuda):
    K, N = 512, 96  # N not a multiple of 128
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=1, device=cuda)
    x = synth.activations(4, K, torch.bfloat16, seed=2, device=cuda)
    with pytest.raises(L.W4Error) as ei:
        ops.nvfp4_gemm(x, w, scale, gscale, act_mode=L.W4_ACT_NVFP4, a_global=_a_global(x))
    assert ei.value.status == L.W4_ERR_UNSUPPORTED


@pytest.mark.parametrize("M", [128, 2048, 4096, 8192])
def test_config3_prefill_sampled_rows(cuda, M):
    """BASELINE config 3 prefill shapes: K=N=5120, activations quantised to NVFP4 on the fly;
    64 sampled rows x all N against the oracle, plus the rows either side of where a call with
    a partly empty last round is split along M (M = 2048: 1792, M = 4096: 3712)."""
    K, N = 5120, 5120
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=0, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=1, device=cuda)
    ag = _a_global(x)
    y = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32, act_mode=L.W4_ACT_NVFP4, a_global=ag)
    edges = torch.tensor([r for r in (0, 1791, 1792, 3711, 3712, M - 1) if r < M])
    rows = torch.cat([torch.randperm(M, generator=torch.Generator().manual_seed(M))[:64], edges])
    rows = torch.unique(rows).to(cuda)
    rf, _ = assert_gemm_close(np_(y[rows]), _oracle(x, w, scale, gscale, ag, rows))
    assert rf < 1e-5, rf


def test_scale_atoms_cached_and_equivalent(cuda):
    """Pre-arranged scale atoms (w4_nvfp4_repack_scales) give the same result as the per-call path."""
    M, K, N = 256, 1024, 256
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=3, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=4, device=cuda)
    ag = _a_global(x)
    y1 = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32, act_mode=L.W4_ACT_NVFP4, a_global=ag)
    assert ops.scale_atoms_cached(scale)
    # the raw [K/16, N] scales through the C ABI (rearranged per call in the workspace)
    c = torch.empty((M, N), dtype=torch.float32, device=cuda)
    need = L.lib().w4_nvfp4_workspace_bytes(M, N, K, L.W4_ACT_NVFP4, L.W4_F32)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)  # the sync area starts zeroed
    L.call("w4_nvfp4_gemm", ops._p(x), ops._p(w), L.W4_NVFP4_NK, ops._p(scale), L.W4_E4M3, ops._p(gscale),
           L.W4_ACT_NVFP4, ops._p(ag), ops._p(c), L.W4_F32, None, M, N, K, ops._p(ws), need, ops._stream(x.device))
    assert torch.equal(y1, c)
    # changing the scales in place invalidates the cached atoms
    scale.view(torch.uint8)[0].copy_(scale.view(torch.uint8)[1])
    assert not ops.scale_atoms_cached(scale)
    y2 = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32, act_mode=L.W4_ACT_NVFP4, a_global=ag)
    assert_gemm_close(np_(y2), _oracle(x, w, scale, gscale, ag))
