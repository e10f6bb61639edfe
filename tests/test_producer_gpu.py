"""Fused producer RMSNorm -> NVFP4 activations (w4_rmsnorm_quant_nvfp4) and the
block-scaled GEMM that consumes it (w4_nvfp4_gemm_q), against the CPU oracle and
against the unfused path (quantise the bf16 RMSNorm output, then w4_nvfp4_gemm).

Inputs whose row sums of squares are exact in fp32 in any order make the normalisation itself order-independent, so
the fused result must equal the oracle bit for bit; N(0, 1) inputs differ from
the sequential host sum only in the last bits of inv, so codes may move by one
E2M1 step in a few places (bounded below).
"""
import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, f32, np_
from xe2x2_b200 import _lib as L
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu


def _atoms_to_rows(atoms, M, K):
    """Scale atoms (512-byte blocks of 128 rows x 4 16-k blocks) -> u8 [rows, K/16]."""
    nb = K // 16
    rows = (M + 127) // 128 * 128
    a = np_(atoms).reshape(rows // 128, nb // 4, 32, 4, 4)  # [tile][kc][r%32][r/32][kb%4]
    return a.transpose(0, 3, 2, 1, 4).reshape(rows, nb)


def _exact_inputs(M, K, dtype, seed):
    """Multiples of 1/8 in [-4, 4] (K <= 8192) or of 1/4 in [-2, 2]: every partial sum of
    squares fits the fp32 mantissa, so any summation order gives the same sum."""
    g = torch.Generator().manual_seed(seed)
    if K <= 8192:
        return (torch.randint(-32, 33, (M, K), generator=g).float() / 8).to(dtype)
    assert 4 * K * 16 < 2**24
    return (torch.randint(-8, 9, (M, K), generator=g).float() / 4).to(dtype)


@pytest.mark.parametrize("M,K,dtype,use_gamma", [
    (1, 5120, torch.bfloat16, False),
    (37, 1024, torch.float16, True),
    (130, 2048, torch.bfloat16, True),
    (3, 17408, torch.bfloat16, True),   # 256 threads, 8 register blocks each
    (2, 40960, torch.float16, False),   # rows too wide for registers: two passes over x
    (600, 2048, torch.bfloat16, True),  # streaming kernel: rows arrive by bulk copy, persistent grid
    (333, 12288, torch.float16, False), # streaming kernel at its widest row
])
def test_producer_bit_exact_on_order_independent_sums(cuda, M, K, dtype, use_gamma):
    x = _exact_inputs(M, K, dtype, seed=M)
    gamma = (torch.randint(1, 9, (K,), generator=torch.Generator().manual_seed(1)).float() / 4).to(dtype) \
        if use_gamma else None
    ag = torch.tensor([0.004], device=cuda)
    act = ops.rmsnorm_quant_nvfp4(x.to(cuda), ag, None if gamma is None else gamma.to(cuda), eps=1e-6)
    codes, sf = O.rmsnorm_nvfp4(f32(x), None if gamma is None else f32(gamma), 1e-6, 0.004)
    assert np.array_equal(np_(act.codes)[:M], codes)
    rows = _atoms_to_rows(act.sf_atoms, M, K)
    assert np.array_equal(rows[:M], sf)
    assert not rows[M:].any() and not np_(act.codes)[M:].any()  # padding rows of the last tile
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_producer_close_on_normal_inputs(cuda):
    M, K = 64, 5120
    x = synth.activations(M, K, torch.bfloat16, seed=5)
    ag = torch.tensor([0.0015], device=cuda)
    act = ops.rmsnorm_quant_nvfp4(x.to(cuda), ag)
    codes, sf = O.rmsnorm_nvfp4(f32(x), None, 1e-6, 0.0015)
    got_c = np_(act.codes)[:M]
    frac = float((got_c != codes).mean())
    assert frac < 2e-3, frac
    got = O.nvfp4_act_dequant(got_c, _atoms_to_rows(act.sf_atoms, M, K)[:M], 0.0015, M, K)
    ref = O.nvfp4_act_dequant(codes, sf, 0.0015, M, K)
    assert float(np.linalg.norm(got - ref) / np.linalg.norm(ref)) < 5e-3


@pytest.mark.parametrize("M,N,K", [(1, 512, 1024), (200, 768, 2048), (1024, 5120, 5120)])
def test_gemm_on_fused_activations_equals_unfused_path(cuda, M, N, K):
    """Exact-sum inputs: the producer's codes equal quant_act of the bf16 RMSNorm
    output, so the two GEMM paths agree bit for bit."""
    x = _exact_inputs(M, K, torch.bfloat16, seed=K)
    ag = torch.tensor([0.003], device=cuda)
    xd = x.to(cuda)
    ss = (x.double() ** 2).sum(1).float()  # exact
    inv = 1.0 / torch.sqrt(ss / K + 1e-6)  # IEEE float32 on the host
    y = (x.float() * inv[:, None]).to(torch.bfloat16).to(cuda)
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=M, device=cuda)
    act = ops.rmsnorm_quant_nvfp4(xd, ag)
    got = ops.nvfp4_gemm_q(act, w, scale, gscale)
    want = ops.nvfp4_gemm(y, w, scale, gscale, act_mode=L.W4_ACT_NVFP4, a_global=ag)
    assert torch.equal(got, want)
    g32 = ops.nvfp4_gemm_q(act, w, scale, gscale, out_dtype=torch.float32)
    q8, rs = ops.nvfp4_gemm_q(act, w, scale, gscale, out_dtype=torch.float8_e4m3fn)
    assert torch.allclose(rs, g32.abs().amax(1) / 448.0, rtol=1e-6)
    rows = slice(0, min(M, 16))
    codes, sf = O.rmsnorm_nvfp4(f32(x[rows]), None, 1e-6, 0.003)
    a_deq = O.nvfp4_act_dequant(codes, sf, 0.003, codes.shape[0], K)
    ref = O.nvfp4_gemm(a_deq, np_(w.contiguous()), O.NVFP4_KN, np_(scale.view(torch.uint8)), O.SCALE_E4M3,
                       float(gscale.item()), a_deq.shape[0], N, K)
    rf, _ = assert_gemm_close(np_(g32[rows]), ref)
    assert rf < 1e-5, rf  # identical operands, fp32 sums
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_producer_argument_errors(cuda):
    ag = torch.tensor([0.01], device=cuda)
    with pytest.raises(ValueError):
        ops.rmsnorm_quant_nvfp4(torch.zeros(2, 96, dtype=torch.bfloat16, device=cuda), ag)  # K % 64
    with pytest.raises(ValueError):
        ops.rmsnorm_quant_nvfp4(torch.zeros(2, 128, device=cuda), ag)  # fp32 input
    lib = L.lib()
    rc = lib.w4_rmsnorm_quant_nvfp4(None, L.W4_BF16, None, 1e-6, None, None, None, 1, 128, None)
    assert rc == L.W4_ERR_INVALID
