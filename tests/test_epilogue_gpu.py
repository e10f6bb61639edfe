"""epilogue_quant parity: fused RMSNorm + s8 and the fp8 row-scale cast."""
import numpy as np
import pytest
import torch

import oracle as O
from tests._util import np_
from xe2x2_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,k", [(1, 5120), (1, 17408), (64, 5120), (64, 17408)])
def test_rmsnorm_quant_s8_reference_contract(cuda, m, k):
    """The reference's check: f16 device input vs the float host oracle, max_abs <= 1
    (kernels/epilogue_quant/rmsnorm_epilogue.cpp:176-204, shapes :268)."""
    x = O.fill_rmsnorm_x(m * k).reshape(m, k)
    q_ref, s_ref = O.rmsnorm_quant_s8(x)
    q, s = ops.rmsnorm_quant_s8(torch.from_numpy(x).to(torch.float16).to(cuda))
    assert int(np.abs(np_(q).astype(np.int32) - q_ref.astype(np.int32)).max()) <= 1
    np.testing.assert_allclose(np_(s), s_ref, rtol=2e-3)


def test_rmsnorm_quant_s8_same_input(cuda):
    """Same f16 input on both sides: only the sum of squares is reduced in a different
    order, so codes agree except at exact rounding boundaries."""
    rng = np.random.default_rng(0)
    x16 = (rng.standard_normal((33, 4096)) * 3).astype(np.float16)
    q_ref, s_ref = O.rmsnorm_quant_s8(x16.astype(np.float32))
    q, s = ops.rmsnorm_quant_s8(torch.from_numpy(x16).to(cuda))
    d = np.abs(np_(q).astype(np.int32) - q_ref.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() < 1e-3
    np.testing.assert_allclose(np_(s), s_ref, rtol=1e-5)


def test_rmsnorm_zero_row(cuda):
    x = torch.zeros((3, 256), dtype=torch.float16, device=cuda)
    x[1] = 1.0
    q, s = ops.rmsnorm_quant_s8(x)
    assert torch.all(q[0] == 0) and s[0].item() == 1.0
    assert torch.all(q[1] == 127)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_rowscale_fp8_bit_exact(cuda, dtype):
    rng = np.random.default_rng(1)
    y = torch.from_numpy((rng.standard_normal((7, 1000)) * 10).astype(np.float32)).to(dtype)
    y[3] = 0
    q, s = ops.rowscale_fp8(y.to(cuda))
    q_ref, s_ref = O.rowscale_fp8(np_(y.float()))
    assert np.array_equal(np_(q.view(torch.uint8)), q_ref)
    assert np.array_equal(np_(s), s_ref)


def _sync_area_zero(dev):
    from xe2x2_b200 import _lib as L
    buf, _ = ops._WS.get(dev, 1)
    return bool((buf[:L.W4_WORKSPACE_SYNC_BYTES] == 0).all())


@pytest.mark.parametrize("M,N,K", [(1, 17408, 5120), (5, 4096, 4096), (16, 5120, 2176)])
def test_gptq_fp8_output_fused_row_max(cuda, M, N, K):
    """Decode sizes: the GEMM folds the row maxima into the workspace and the cast reads its f32
    product once.  The fp8 codes and row scales equal the two-pass cast of the same call's f32
    output bit for bit, twice in a row, and the sync area is zero again afterwards."""
    from xe2x2_b200 import synth
    qw, qz, sc, _ = synth.gptq_weights(K, N, 128, asym=True, seed=M, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=M + 1, device=cuda)
    y = ops.gptq_gemm(a, qw, qz, sc, 128, 1, out_dtype=torch.float32)
    q_ref, s_ref = O.rowscale_fp8(np_(y))
    for _ in range(2):
        q, s = ops.gptq_gemm(a, qw, qz, sc, 128, 1, out_dtype=torch.float8_e4m3fn)
        torch.cuda.synchronize()
        assert np.array_equal(np_(q.view(torch.uint8)), q_ref)
        assert np.array_equal(np_(s), s_ref)
        assert _sync_area_zero(cuda)


@pytest.mark.parametrize("M", [1, 8])
def test_nvfp4_fp8_output_fused_row_max(cuda, M):
    """The same for the NVFP4 W4A16 decode GEMM."""
    from xe2x2_b200 import synth
    K, N = 5120, 5120
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=M, device=cuda)
    x = synth.activations(M, K, torch.bfloat16, seed=M + 2, device=cuda)
    y = ops.nvfp4_gemm(x, w, scale, gscale, torch.float32)
    q_ref, s_ref = O.rowscale_fp8(np_(y))
    for _ in range(2):
        q, s = ops.nvfp4_gemm(x, w, scale, gscale, torch.float8_e4m3fn)
        torch.cuda.synchronize()
        assert np.array_equal(np_(q.view(torch.uint8)), q_ref)
        assert np.array_equal(np_(s), s_ref)
        assert _sync_area_zero(cuda)
