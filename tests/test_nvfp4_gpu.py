"""NVFP4 parity: CUDA path (through the C ABI) vs the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, bits16, f32, np_
from xe2x2_b200 import _lib as L
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu


def _w_kn_np(w):
    """u8 [K/2, N] logical view -> numpy KN array."""
    return np_(w.contiguous())


def _oracle_gemm(x, w, scale, gscale):
    K, N = w.shape[0] * 2, w.shape[1]
    kind = O.SCALE_E4M3 if scale.dtype == torch.float8_e4m3fn else O.SCALE_BF16
    sc = np_(scale.view(torch.uint8)) if kind == O.SCALE_E4M3 else bits16(scale)
    g = float(gscale.item()) if gscale is not None else 1.0
    return O.nvfp4_gemm(f32(x), _w_kn_np(w), O.NVFP4_KN, sc, kind, g, x.shape[0], N, K)


def _subnormal_scales(scale):
    s = scale.view(torch.uint8).clone()
    s[::7, ::5] = torch.randint(1, 8, s[::7, ::5].shape, dtype=torch.uint8, device=s.device)  # e4m3 subnormals
    s[3, :] = 0  # zero block scale
    return s.view(torch.float8_e4m3fn)


@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_dequant_bit_exact(cuda, layout):
    K, N = 512, 96
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=3, device=cuda)
    scale = _subnormal_scales(scale)
    if layout == "kn":
        w = w.contiguous()
    got = ops.nvfp4_dequant(w, scale, gscale)
    ref = O.nvfp4_dequant(_w_kn_np(w), O.NVFP4_KN, np_(scale.view(torch.uint8)), O.SCALE_E4M3,
                          float(gscale.item()), K, N)
    assert np.array_equal(np_(got), ref)


def test_dequant_bf16_scale_bit_exact(cuda):
    K, N = 256, 64
    w, _, _ = synth.nvfp4_weights(K, N, seed=4, device=cuda)
    scale = (torch.rand((K // 16, N), device=cuda) * 0.05).to(torch.bfloat16)
    got = ops.nvfp4_dequant(w, scale, None)
    ref = O.nvfp4_dequant(_w_kn_np(w), O.NVFP4_KN, bits16(scale), O.SCALE_BF16, 1.0, K, N)
    assert np.array_equal(np_(got), ref)


def test_repack_kn_to_nk_exact(cuda):
    K, N = 640, 160
    g = torch.Generator(device=cuda).manual_seed(1)
    w_kn = torch.randint(0, 256, (K // 2, N), dtype=torch.uint8, device=cuda, generator=g)
    w_nk = ops.nvfp4_repack_kn_to_nk(w_kn)
    assert w_nk.stride(0) == 1 and torch.equal(w_nk, w_kn)


def test_quant_act_bit_exact(cuda):
    M, K = 9, 1024
    x = synth.activations(M, K, torch.bfloat16, seed=5, device=cuda)
    x[2, 16:32] = 0  # an all-zero block
    x[4, :8] *= 1000.0  # saturating block
    amax = float(x.abs().max().float().item())
    a_global = torch.tensor([amax / (448.0 * 6.0)], dtype=torch.float32, device=cuda)
    codes, sf = ops.nvfp4_quant_act(x, a_global)
    rc, rs = O.nvfp4_quant_act(f32(x), float(a_global.item()))
    assert np.array_equal(np_(codes), rc)
    assert np.array_equal(np_(sf), rs)


def test_quant_act_rounding_ties_bit_exact(cuda):
    """Values that land exactly on E2M1 midpoints (ties to even), negative values
    that round to zero, and saturation: with a_global = 1 and a block maximum of 6
    the block scale decodes to 1, so every element is quantised as is."""
    K = 64
    row = [6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -0.1,
           6.0, 0.2, 0.3, 0.74, 0.76, 1.24, 1.26, 2.49, 2.51, 3.49, 3.51, 4.99, 5.01, -0.0, 0.0, -6.0,
           6.0, 7.0, -7.0, 1e-3, -1e-3, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, -0.5, -1.0, -1.5, -2.0, -3.0,
           6.0, -4.0, 0.125, 0.375, 0.625, 0.875, 1.125, 1.375, 2.25, 2.75, 3.25, 3.75, 4.5, 5.5, 5.75, 0.0]
    x = torch.tensor([row, [v * 0.5 for v in row]], dtype=torch.float32).to(torch.bfloat16).to(cuda)
    a_global = torch.ones(1, dtype=torch.float32, device=cuda)
    codes, sf = ops.nvfp4_quant_act(x, a_global)
    rc, rs = O.nvfp4_quant_act(f32(x), 1.0)
    assert np.array_equal(np_(sf), rs)
    assert np.array_equal(np_(codes), rc)


@pytest.mark.parametrize("M", [1, 2, 5, 8, 16, 17, 32, 40])
def test_gemm_w4a16_small(cuda, M):
    K, N = 1024, 256
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=M, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=M + 1, device=cuda)
    out = ops.nvfp4_gemm_w4a16_f8scale(x, w, None, scale, gscale, 16)
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    assert_gemm_close(f32(out), _oracle_gemm(x, w, scale, gscale))


def test_gemm_w4a16_exact_weights_fp32_out(cuda):
    """e2m1 * e4m3 (incl. subnormal and zero scales) is exact in bf16: fp32 out matches to rounding."""
    M, K, N = 4, 2048, 128
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=8, device=cuda)
    scale = _subnormal_scales(scale)
    x = synth.activations(M, K, torch.bfloat16, seed=9, device=cuda)
    out = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32)
    assert_gemm_close(np_(out), _oracle_gemm(x, w, scale, gscale), rel=1e-5, nmax=1e-5)


@pytest.mark.parametrize("M", [1, 16])
def test_config3_decode(cuda, M):
    """BASELINE config 3 decode shapes: K=N=5120."""
    K, N = 5120, 5120
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=0, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=1, device=cuda)
    ops.register_torch_ops()
    out = torch.ops.w4.nvfp4_gemm_w4a16_f8scale(x, w, None, scale, gscale, 16)
    rf, _ = assert_gemm_close(f32(out), _oracle_gemm(x, w, scale, gscale))
    assert rf < 5e-3


@pytest.mark.parametrize("M", [3, 12, 40])
def test_bf16_folded_scale_operator(cuda, M):
    """nvfp4_gemm_w4a16(x, w, None, scale_bf16, 16): folded scales, weights rounded to bf16
    (always the decode kernels, two token tiles from M = 9)."""
    K, N = 1024, 128
    w, _, _ = synth.nvfp4_weights(K, N, seed=6, device=cuda)
    scale = (torch.rand((K // 16, N), device=cuda) * 0.05 + 0.001).to(torch.bfloat16)
    x = synth.activations(M, K, torch.bfloat16, seed=7, device=cuda)
    out = ops.nvfp4_gemm_w4a16(x, w, None, scale, 16)
    assert_gemm_close(f32(out), _oracle_gemm(x, w, scale, None))


def test_two_token_tile_decode_on_shapes_the_tensor_path_skips(cuda):
    """N % 128 != 0 keeps M = 9..16 on the two-token-tile decode kernel."""
    M, K, N = 12, 1024, 96
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=12, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=13, device=cuda)
    out = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32)
    assert_gemm_close(np_(out), _oracle_gemm(x, w, scale, gscale), rel=1e-5, nmax=1e-5)


def test_kn_weights_accepted_by_operator(cuda):
    M, K, N = 2, 512, 64
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=2, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, device=cuda)
    a = ops.nvfp4_gemm(x, w, scale, gscale)
    b = ops.nvfp4_gemm(x, w.contiguous(), scale, gscale)
    assert torch.equal(a, b)


def test_fp8_rowscale_output(cuda):
    M, K, N = 5, 1024, 256
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=12, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=13, device=cuda)
    y = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32)
    q, rs = ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float8_e4m3fn)
    q_ref, s_ref = O.rowscale_fp8(np_(y))
    assert np.array_equal(np_(q.view(torch.uint8)), q_ref)
    assert np.array_equal(np_(rs), s_ref)


def test_lut_reference_formula_bit_exact(cuda):
    """w4_nvfp4_lut_gemm_s8a reproduces nibble_lut_sc.cpp:319-330 bit for bit."""
    for rows, k, cols in [(4, 64, 32), (4, 1024, 256), (1, 5120, 512)]:
        a = O.fill_s8(rows * k, 1).reshape(rows, k)
        nib = O.fill_nibbles(k * cols, 9).reshape(k, cols)
        packed = ((nib[0::2] & 15) | ((nib[1::2] & 15) << 4)).astype(np.uint8)
        a_s = np.full(rows, 0.02, np.float32)
        b_s = np.full(cols, 0.02, np.float32)
        got = ops.nvfp4_lut_gemm_s8a(torch.from_numpy(a).to(cuda), torch.from_numpy(packed).to(cuda),
                                     torch.from_numpy(a_s).to(cuda), torch.from_numpy(b_s).to(cuda), rows, cols, k)
        ref = O.nvfp4_lut_gemm_s8a(a, packed, a_s, b_s)
        assert np.array_equal(bits16(got), ref)


def test_errors(cuda):
    w, scale, gscale = synth.nvfp4_weights(256, 64, seed=1, device=cuda)
    x = synth.activations(1, 256, torch.bfloat16, device=cuda)
    with pytest.raises(L.W4Error) as e:
        ops.nvfp4_gemm(x[:, :200].contiguous(), synth.nvfp4_weights(200, 64, device=cuda)[0],
                       torch.ones((12, 64), device=cuda).to(torch.float8_e4m3fn), gscale)
    assert e.value.status in (L.W4_ERR_INVALID, L.W4_ERR_UNSUPPORTED)
    with pytest.raises(ValueError):
        ops.nvfp4_gemm_w4a16_f8scale(x, w, None, scale, gscale, 32)
