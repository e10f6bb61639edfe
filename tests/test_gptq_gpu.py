"""GPTQ int4 parity: CUDA path (through the C ABI) vs the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, bits16, f32, np_
from xe2x2_b200 import _lib as L
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu


def _oracle_gemm(a, qw, qz, sc, g_idx, K, N, gs, zo):
    return O.gptq_gemm(f32(a), np_(qw), None if qz is None else np_(qz), bits16(sc),
                       None if g_idx is None else np_(g_idx), a.shape[0], N, K, gs, zo)


@pytest.mark.parametrize("asym,zo,gs,act", [(True, 1, 128, False), (True, 0, 64, False), (False, 1, 128, False),
                                            (True, 1, 32, False), (True, 1, 128, True)])
def test_dequant_bit_exact(cuda, asym, zo, gs, act):
    K, N = 1024, 384
    qw, qz, sc, gi = synth.gptq_weights(K, N, gs, asym=asym, seed=7, device=cuda, act_order=act)
    got = ops.gptq_dequant(qw, qz, sc, gi, gs, zo)
    ref = O.gptq_dequant(np_(qw), None if qz is None else np_(qz), bits16(sc),
                         None if gi is None else np_(gi), K, N, gs, zo)
    assert np.array_equal(np_(got), ref)


@pytest.mark.parametrize("M", [1, 3, 4, 8, 9, 16, 17, 32, 33, 70])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gemm_small_shapes(cuda, M, dtype):
    K, N, gs = 1024, 256, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=M, device=cuda)
    a = synth.activations(M, K, dtype, seed=M + 100, device=cuda)
    out = ops.gptq_gemm(a, qw, qz, sc, gs, 1)
    assert out.dtype == dtype and out.shape == (M, N)
    assert_gemm_close(f32(out), _oracle_gemm(a, qw, qz, sc, None, K, N, gs, 1))


@pytest.mark.parametrize("gs,zo,asym", [(32, 1, True), (64, 0, True), (128, 1, False), (256, 1, True)])
def test_gemm_group_sizes_and_zero_conventions(cuda, gs, zo, asym):
    M, K, N = 5, 2048, 512
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=asym, seed=gs, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=11, device=cuda)
    out = ops.gptq_gemm(a, qw, qz, sc, gs, zo, out_dtype=torch.float32)
    assert_gemm_close(np_(out), _oracle_gemm(a, qw, qz, sc, None, K, N, gs, zo), rel=1e-4, nmax=1e-4)


def test_config1_full_size(cuda):
    """M=16, K=N=4096, g128, symmetric, fp16 in/out."""
    M, K, N, gs = 16, 4096, 4096, 128
    qw, _, sc, _ = synth.gptq_weights(K, N, gs, asym=False, seed=0, device=cuda)
    a = synth.activations(M, K, torch.float16, seed=1, device=cuda)
    out = ops.gptq_gemm(a, qw, None, sc, gs, 1)
    rf, _ = assert_gemm_close(f32(out), _oracle_gemm(a, qw, None, sc, None, K, N, gs, 1))
    assert rf < 2e-3
    # stored zero 7 with the v1 "+1" convention is the same layer
    qz7 = torch.full((K // gs, N // 8), 0x77777777, dtype=torch.int32, device=cuda)
    out7 = ops.gptq_gemm(a, qw, qz7, sc, gs, 1)
    assert torch.equal(out, out7)


@pytest.mark.parametrize("M", [1, 4, 8, 16])
def test_config2_decode_sweep(cuda, M):
    """K=5120, N=17408, g128, asymmetric, bf16 in/out."""
    K, N, gs = 5120, 17408, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=0, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=1, device=cuda)
    out = ops.gptq_gemm(a, qw, qz, sc, gs, 1)
    rf, _ = assert_gemm_close(f32(out), _oracle_gemm(a, qw, qz, sc, None, K, N, gs, 1))
    assert rf < 5e-3


def test_act_order_repack_and_gemm(cuda):
    M, K, N, gs = 7, 2048, 256, 128
    qw, qz, sc, gi = synth.gptq_weights(K, N, gs, asym=True, seed=5, device=cuda, act_order=True)
    lin = ops.GPTQLinear(qw, qz, sc, gi, gs, 1)
    assert lin.perm is not None
    assert np.array_equal(np_(lin.perm), O.gptq_act_order_perm(np_(gi), gs))
    # repacked codes: row j of the new matrix is row perm[j] of the old one
    u_old = O.unpack_i32_nibbles_first(np_(qw))
    u_new = O.unpack_i32_nibbles_first(np_(lin.qweight))
    assert np.array_equal(u_new, u_old[np_(lin.perm)])
    a = synth.activations(M, K, torch.bfloat16, seed=6, device=cuda)
    out = lin(a, out_dtype=torch.float32)
    assert_gemm_close(np_(out), _oracle_gemm(a, qw, qz, sc, gi, K, N, gs, 1), rel=1e-4, nmax=1e-4)


def test_act_order_rejects_unequal_groups(cuda):
    K, N, gs = 256, 64, 128
    qw, _, _, _ = synth.gptq_weights(K, N, gs, asym=False, seed=1, device=cuda)
    g_idx = torch.zeros(K, dtype=torch.int32, device=cuda)  # all rows in group 0
    with pytest.raises(L.W4Error) as e:
        ops.gptq_repack_act_order(qw, g_idx, gs)
    assert e.value.status == L.W4_ERR_UNSUPPORTED


def test_fp8_rowscale_output(cuda):
    M, K, N, gs = 6, 1024, 512, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=9, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=10, device=cuda)
    y = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float32)
    q, rs = ops.gptq_gemm(a, qw, qz, sc, gs, 1, out_dtype=torch.float8_e4m3fn)
    q_ref, s_ref = O.rowscale_fp8(np_(y))  # the cast itself is bit-exact given the same y
    assert np.array_equal(np_(q.view(torch.uint8)), q_ref)
    assert np.array_equal(np_(rs), s_ref)
    # and the dequantised fp8 output tracks the oracle GEMM within fp8 precision
    deq = f32(q) * np_(rs)[:, None]
    assert_gemm_close(deq, _oracle_gemm(a, qw, qz, sc, None, K, N, gs, 1), rel=5e-2, nmax=7e-2)


def test_s4a_reference_formula_bit_exact(cuda):
    """w4_gptq_gemm_s4a reproduces dpas_s4_gptq_sc.cpp:273-288 bit for bit."""
    for rows, k, cols in [(8, 128, 16), (8, 256, 256), (4, 5120, 1024), (1, 1024, 4096)]:
        a, b, asc, s = synth.gptq_s4_tile(rows, k, cols, seed=rows + k)
        ad = torch.from_numpy(O.pack_s4_rows(np_(a))).to(cuda)
        bd = torch.from_numpy(O.pack_s4_along_k(np_(b))).to(cuda)
        got = ops.gptq_gemm_s4a(ad, bd, asc.to(cuda), s.to(cuda), rows, cols, k)
        ref = O.gptq_s4a_gemm(np_(a), np_(asc), np_(b), bits16(s), 128)
        assert np.array_equal(bits16(got), ref)


def test_deterministic_and_stream_ordered(cuda):
    M, K, N, gs = 16, 4096, 1024, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=3, device=cuda)
    a = synth.activations(M, K, torch.bfloat16, seed=4, device=cuda)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        o1 = ops.gptq_gemm(a, qw, qz, sc, gs, 1)
        o2 = ops.gptq_gemm(a, qw, qz, sc, gs, 1)
    s.synchronize()
    assert torch.equal(o1, o2)


def test_errors_are_raised(cuda):
    qw, qz, sc, _ = synth.gptq_weights(256, 64, 128, seed=1, device=cuda)
    a = synth.activations(2, 256, torch.bfloat16, device=cuda)
    with pytest.raises(L.W4Error) as e:
        ops.gptq_gemm(a, qw, qz, sc, 96, 1)  # K % group_size != 0
    assert e.value.status == L.W4_ERR_INVALID
    with pytest.raises(ValueError):
        ops.gptq_gemm(a.cpu(), qw, qz, sc, 128, 1)  # no CPU path


def test_torch_op_registration(cuda):
    ops.register_torch_ops()
    M, K, N, gs = 3, 512, 128, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, seed=2, device=cuda)
    a = synth.activations(M, K, torch.float16, device=cuda)
    out = torch.ops.w4.gptq_gemm(a, qw, qz, sc, None, gs, 1)
    assert torch.equal(out, ops.gptq_gemm(a, qw, qz, sc, gs, 1))


def test_out_argument_writes_in_place(cuda):
    K, N, gs = 1024, 256, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=31, device=cuda)
    a = synth.activations(24, K, torch.bfloat16, seed=32, device=cuda)
    buf = torch.full((30, N), float("nan"), dtype=torch.bfloat16, device=cuda)
    ref = ops.gptq_gemm(a, qw, qz, sc, gs, 1)
    got = ops.gptq_gemm(a[:8], qw, qz, sc, gs, 1, out=buf[2:10])
    assert got.data_ptr() == buf[2:10].data_ptr()
    assert torch.equal(buf[2:10], ops.gptq_gemm(a[:8].contiguous(), qw, qz, sc, gs, 1))
    assert torch.isnan(buf[:2].float()).all() and torch.isnan(buf[10:].float()).all()
    ops.gptq_gemm(a, qw, qz, sc, gs, 1, out=buf[4:28])
    assert torch.equal(buf[4:28], ref)
    with pytest.raises(ValueError):
        ops.gptq_gemm(a, qw, qz, sc, gs, 1, out=buf[:10])
