"""GPTQ prefill GEMM (tcgen05 tensor-core path, M >= 17) vs the CPU oracle.

The weights reach the tensor core as bf16 (or f16) values (q - z) * s rounded
once, so the tolerance is the north-star contract (rel Frobenius 1e-2, max-abs
2e-2 after normalisation) with a tighter expectation checked alongside.
"""
import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, bits16, f32, np_
from xe2x2_b200 import _lib as L
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu


def _oracle(a, qw, qz, sc, K, N, gs, zo=1, g_idx=None):
    return O.gptq_gemm(f32(a), np_(qw), None if qz is None else np_(qz), bits16(sc),
                       None if g_idx is None else np_(g_idx), a.shape[0], N, K, gs, zo)


@pytest.mark.parametrize("M,K,N,gs,asym,dtype,out", [
    (17, 512, 256, 128, True, torch.bfloat16, torch.float32),     # M tail, 256-wide tiles
    (128, 1024, 384, 64, True, torch.bfloat16, torch.bfloat16),   # 128-wide tiles (N % 256 != 0), g64
    (200, 2048, 512, 128, False, torch.float16, torch.float16),   # symmetric, f16 path
    (300, 1024, 768, 128, True, torch.bfloat16, torch.float32),   # three M tiles, mixed tile widths
    (64, 4096, 256, 256, True, torch.float16, torch.float32),     # group 256
    (64, 2688, 1856, 128, True, torch.bfloat16, torch.float32),   # N % 128 != 0: ragged last tile
    (40, 1856, 2688, 64, True, torch.bfloat16, torch.bfloat16),   # 2688 = 10.5 x 256
    (24, 1024, 96, 128, True, torch.bfloat16, torch.float32),     # N below one tile
])
def test_prefill_shapes(cuda, M, K, N, gs, asym, dtype, out):
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=asym, seed=M + N, device=cuda)
    a = synth.activations(M, K, dtype, seed=M, device=cuda)
    got = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=out)
    assert got.dtype == out and got.shape == (M, N)
    rf, _ = assert_gemm_close(f32(got), _oracle(a, qw, qz, sc, K, N, gs))
    assert rf < 4e-3, rf  # one bf16 rounding per weight
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_prefill_zero_offset_v2(cuda):
    M, K, N, gs = 96, 1024, 256, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=3, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=4, device=cuda)
    got = ops.gptq_gemm(a, qw, qz, sc, gs, 0, out_dtype=torch.float32)
    assert_gemm_close(np_(got), _oracle(a, qw, qz, sc, K, N, gs, zo=0))


def test_prefill_fp8_rowscale(cuda):
    M, K, N, gs = 130, 1024, 512, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=9, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=10, device=cuda)
    q8, rs = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float8_e4m3fn)
    ref = _oracle(a, qw, qz, sc, K, N, gs)
    assert np.allclose(np_(rs), np.abs(ref).max(axis=1) / 448.0, rtol=1e-2)
    assert_gemm_close(np_(q8.float() * rs[:, None]), ref, rel=4e-2, nmax=8e-2)


def test_prefill_matches_decode_path_on_boundary(cuda):
    """M=16 runs the decode GEMV, M=17 the tensor-core GEMM: the shared rows agree."""
    K, N, gs = 2048, 512, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=21, device=cuda)
    a = synth.activations(17, K, torch.bfloat16, seed=22, device=cuda)
    y17 = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float32)
    y16 = ops.gptq_gemm(a[:16].contiguous(), qw, qz, sc, gs, 1, out_dtype=torch.float32)
    rel = float((y17[:16] - y16).norm() / y16.norm())
    assert rel < 4e-3, rel


def test_config4_act_order_sampled_rows(cuda):
    """BASELINE config 4 at full size: M=2048, K=5120, N=27648, g128, act_order,
    asymmetric zeros, A ~ N(0, 0.5); 64 sampled rows x all N checked against the oracle."""
    M, K, N, gs = 2048, 5120, 27648, 128
    qw, qz, sc, gi = synth.gptq_weights(K, N, gs, asym=True, seed=0, device=cuda, act_order=True)
    a = synth.activations(M, K, torch.bfloat16, sigma=0.5, seed=1, device=cuda)
    lin = ops.GPTQLinear(qw, qz, sc, gi, gs, 1)
    y = lin(a)
    torch.cuda.synchronize()
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(0))[:64].sort().values
    ref = _oracle(a[rows.to(cuda)], qw, qz, sc, K, N, gs, g_idx=gi)
    rf, _ = assert_gemm_close(f32(y[rows.to(cuda)]), ref)
    assert rf < 4e-3, rf
    assert L.lib().w4_check_device_status() == L.W4_OK


@pytest.mark.parametrize("M,K,N", [(32, 17408, 5120), (64, 5120, 7168), (48, 2176, 5120), (200, 4096, 640), (17, 8192, 256)])
def test_prefill_split_k(cuda, M, K, N):
    """Few output tiles: the tensor-core GEMM splits K across CTAs and sums fp32 partials
    (tensor-parallel down / o projection shapes)."""
    gs = 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=K + M, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=M, device=cuda)
    assert L.lib().w4_gptq_workspace_bytes(M, N, K, gs, 0, L.W4_BF16) > 0  # partials are needed
    got = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float32)
    rf, _ = assert_gemm_close(np_(got), _oracle(a, qw, qz, sc, K, N, gs))
    assert rf < 4e-3, rf
    got16 = ops.gptq_gemm(a, qw, qz, sc, gs, 1)
    assert_gemm_close(f32(got16), _oracle(a, qw, qz, sc, K, N, gs))
