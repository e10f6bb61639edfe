"""Size-independent properties at BASELINE's full sizes, where the CPU oracle would take
too long: every path accumulates exact products in fp32 in a fixed order, so

* scaling the activations by 2 scales the fp32 output by exactly 2 (bit for bit), and
* permuting the rows of the activations permutes the output rows (bit for bit), except
  where a call runs as two along M (a tensor-core GEMM whose last wave would be mostly empty:
  its last rows are split along K, another fp32 order): there rows computed in the first part
  both times are bit-identical and the rest agree to fp32 summation order.

For the NVFP4-activation path the tensor scale a_global is doubled with the
activations, so the codes and block scales are unchanged and only the final tensor
scale doubles.
"""
import pytest
import torch

from xe2x2_b200 import _lib as L
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu


def _check_linear_and_row_independent(f, a, split_at=None):
    y = f(a)
    assert torch.equal(f(a * 2), y * 2)
    perm = torch.randperm(a.shape[0], generator=torch.Generator().manual_seed(0)).to(a.device)
    yp = f(a[perm].contiguous())
    if split_at is None:
        assert torch.equal(yp, y[perm])
    else:  # rows [split_at, M) of a call are K-split: compare them to fp32 summation order
        both = (perm < split_at) & (torch.arange(a.shape[0], device=a.device) < split_at)
        assert torch.equal(yp[both], y[perm][both])
        rel = float((yp - y[perm]).norm() / y.norm())
        assert rel < 1e-5, rel
    assert torch.isfinite(y).all()


@pytest.mark.parametrize("M", [1, 16])
def test_config2_decode_properties(cuda, M):
    K, N, gs = 5120, 17408, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=0, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=1, device=cuda)
    _check_linear_and_row_independent(lambda x: ops.gptq_gemm(x, qw, qz, sc, gs, 1, out_dtype=torch.float32), a)
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_config4_prefill_act_order_properties(cuda):
    M, K, N, gs = 2048, 5120, 27648, 128
    qw, qz, sc, gi = synth.gptq_weights(K, N, gs, asym=True, seed=0, device=cuda, act_order=True)
    lin = ops.GPTQLinear(qw, qz, sc, gi, gs, 1)
    a = synth.activations(M, K, torch.bfloat16, sigma=0.5, seed=1, device=cuda)
    _check_linear_and_row_independent(lambda x: lin(x, out_dtype=torch.float32), a)
    assert L.lib().w4_check_device_status() == L.W4_OK


@pytest.mark.parametrize("M", [1, 2048])
def test_config3_w4a16_properties(cuda, M):
    K = N = 5120
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=0, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=1, device=cuda)
    # M = 2048: 160 tiles of 256 x 256 for 148 SMs, run as rows [0, 1792) and [1792, 2048)
    _check_linear_and_row_independent(lambda x: ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32), a,
                                      split_at=1792 if M == 2048 else None)
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_config3_nvfp4_activation_properties(cuda):
    M, K, N = 2048, 5120, 5120
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=0, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=1, device=cuda)
    ag = torch.tensor([float(a.float().abs().max()) / 2688.0], device=cuda)

    def f(x, g):
        return ops.nvfp4_gemm(x, w, scale, gscale, out_dtype=torch.float32, act_mode=L.W4_ACT_NVFP4, a_global=g)

    y = f(a, ag)
    assert torch.equal(f(a * 2, ag * 2), y * 2)
    perm = torch.randperm(M, generator=torch.Generator().manual_seed(0)).to(cuda)
    assert torch.equal(f(a[perm].contiguous(), ag), y[perm])
    assert L.lib().w4_check_device_status() == L.W4_OK
