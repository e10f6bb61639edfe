"""NVFP4 weights with bf16 activations from 9 tokens on: the tcgen05
tensor-core GEMM with in-shared-memory dequantisation, against the CPU oracle.

Every weight e2m1 * e4m3 is exact in bf16, so with fp32 output the only
difference from the oracle is the fp32 summation order (rel <= 1e-5)."""
import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, f32, np_
from xe2x2_b200 import _lib as L
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu


def _oracle(x, w, scale, gscale):
    K, N = w.shape[0] * 2, w.shape[1]
    return O.nvfp4_gemm(f32(x), np_(w.contiguous()), O.NVFP4_KN, np_(scale.view(torch.uint8)), O.SCALE_E4M3,
                        float(gscale.item()), x.shape[0], N, K)


@pytest.mark.parametrize("M,K,N", [
    (9, 512, 256),       # first tensor-core size, 256-wide tiles
    (17, 512, 256),
    (128, 1024, 384),    # 128-wide tiles (N % 256 != 0)
    (300, 2048, 512),    # three 128-row tiles: two A tiles per CTA
    (32, 8192, 256),     # few output tiles: K split across CTAs
    (40, 2688, 1856),    # N % 128 != 0: ragged last tile
    (24, 1920, 2688),    # 2688 = 10.5 x 256
])
def test_w4a16_prefill_matches_oracle(cuda, M, K, N):
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=M + K, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=M, device=cuda)
    got = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32)
    rf, _ = assert_gemm_close(np_(got), _oracle(x, w, scale, gscale))
    assert rf < 1e-5, rf
    b16 = ops.nvfp4_gemm(x, w, scale, gscale)
    assert_gemm_close(f32(b16), _oracle(x, w, scale, gscale))
    q8, rs = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float8_e4m3fn)
    assert torch.allclose(rs, got.abs().amax(1) / 448.0, rtol=1e-6)
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_w4a16_boundary_decode_and_prefill_agree(cuda):
    """M=8 runs the decode GEMV, M=9 the tensor-core GEMM: the shared rows agree."""
    K, N = 2048, 512
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=5, device=cuda)
    x = synth.activations(9, K, torch.bfloat16, seed=6, device=cuda)
    y9 = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32)
    y8 = ops.nvfp4_gemm(x[:8].contiguous(), w, scale, gscale, out_dtype=torch.float32)
    assert float((y9[:8] - y8).norm() / y8.norm()) < 1e-5


def test_reference_operator_at_prefill_size(cuda):
    """The drop-in operator nvfp4_gemm_w4a16_f8scale (bench_nvfp4_m1.py:88) at config 3 M=2048,
    K=N=5120; 32 sampled rows against the oracle."""
    M, K, N = 2048, 5120, 5120
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=0, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=1, device=cuda)
    y = ops.nvfp4_gemm_w4a16_f8scale(x, w, None, scale, gscale, 16)
    torch.cuda.synchronize()
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(0))[:32].sort().values.to(cuda)
    assert_gemm_close(f32(y[rows]), _oracle(x[rows], w, scale, gscale))
    assert L.lib().w4_check_device_status() == L.W4_OK
