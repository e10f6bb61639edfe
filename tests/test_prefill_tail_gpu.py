"""A prefill GEMM whose tiles leave the last wave partly empty runs as two calls along M (the
row blocks filling whole waves, then the rest with a K split).  The rows of the first part are
bit-identical to the same GEMM run as one call with the same tiling (W4_PREFILL forces that
plan and disables the split); the rest agree to fp32 summation order; sampled rows of both
parts match the host oracle."""
import os

import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, bits16, f32, np_
from xe2x2_b200 import _lib as L, ops, synth

pytestmark = pytest.mark.gpu

M, K, N = 2048, 5120, 5120  # 160 tiles of 256 x 256: 1.08 waves on 148 SMs
M1 = 1792                   # the seven row blocks that fill one wave
ROWS = [0, 1, M1 - 1, M1, M1 + 1, M - 1]


def _forced_whole(fn):
    os.environ["W4_PREFILL"] = "1,1"
    try:
        return fn()
    finally:
        os.environ.pop("W4_PREFILL", None)


def _split_checks(got, whole):
    assert torch.equal(got[:M1], whole[:M1])
    rel = float((got - whole).norm() / whole.norm())
    assert rel < 1e-5, rel  # the tail's K split sums in another fp32 order
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_nvfp4_w4a16_tail_split(cuda):
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=21, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=22, device=cuda)
    got = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32)
    whole = _forced_whole(lambda: ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32))
    _split_checks(got, whole)
    ref = O.nvfp4_gemm(f32(x[ROWS]), np_(w), O.NVFP4_KN, np_(scale.view(torch.uint8)), O.SCALE_E4M3,
                       float(gscale.item()), len(ROWS), N, K)
    rf, _ = assert_gemm_close(np_(got[ROWS]), ref)
    assert rf < 1e-5, rf


def test_gptq_tail_split(cuda):
    gs = 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=23, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=24, device=cuda)
    got = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float32)
    whole = _forced_whole(lambda: ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float32))
    _split_checks(got, whole)
    ref = O.gptq_gemm(f32(a[ROWS]), np_(qw), np_(qz), bits16(sc), None, len(ROWS), N, K, gs, 1)
    rf, _ = assert_gemm_close(np_(got[ROWS]), ref)
    assert rf < 4e-3, rf  # one bf16 rounding per weight
    b16 = ops.gptq_gemm(a, qw, qz, sc, gs, 1)
    assert np.allclose(f32(b16[M1:]), np_(got[M1:]), rtol=1e-2, atol=1e-2 * float(got.abs().max()))
