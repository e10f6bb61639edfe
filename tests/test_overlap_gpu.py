"""Programmatic dependent launch of the decode GEMMs (w4_set_launch_overlap).

Under every overlap mode a decode GEMM must see the complete output of the
kernel launched just before it on the stream: its activations produced by a
torch kernel, or by the previous decode GEMM (GEMM -> GEMM chains, eagerly and
replayed from a CUDA graph).  Results are bit-identical to plain launches.
W4_OVERLAP_DEPENDENT must also see weights written by the preceding kernel.
"""
import pytest
import torch

from xe2x2_b200 import _lib as L
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu

MODES = (L.W4_OVERLAP_OFF, L.W4_OVERLAP_DEPENDENT, L.W4_OVERLAP_STATIC_WEIGHTS)


@pytest.fixture
def overlap_mode():
    old = L.lib().w4_get_launch_overlap()
    yield lambda m: L.call("w4_set_launch_overlap", m)
    L.call("w4_set_launch_overlap", old)


def _gptq_chain(x, layers, gs):
    y = x
    for i, (qw, qz, sc) in enumerate(layers):
        if i % 2:
            y = y * 0.5 + 0.25  # a torch kernel writes the next GEMM's activations
        y = ops.gptq_gemm(y, qw, qz, sc, gs, 1)
        y = y / y.float().abs().amax().clamp_min(1e-6).to(y.dtype)
    return y


def _fp4_chain(x, layers):
    y = x
    for i, (w, s, g) in enumerate(layers):
        y = ops.nvfp4_gemm(y, w, s, g)
        if i % 2:
            y = y / y.float().abs().amax().clamp_min(1e-6).to(y.dtype)
    return y


def _run_modes(fn, set_mode):
    outs = {}
    for m in MODES:
        set_mode(m)
        eager = fn()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            fn()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                replayed = fn()
        torch.cuda.current_stream().wait_stream(st)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        outs[m] = (eager.clone(), replayed.clone())
        del g
    base = outs[L.W4_OVERLAP_OFF][0]
    for m, (e, r) in outs.items():
        assert torch.equal(e, base), m
        assert torch.equal(r, base), m
    assert L.lib().w4_check_device_status() == L.W4_OK


@pytest.mark.parametrize("M", [1, 16])
def test_gptq_decode_chain_identical_under_every_mode(cuda, overlap_mode, M):
    K = N = 2048
    gs = 128
    layers = [synth.gptq_weights(K, N, gs, asym=True, seed=40 + i, device=cuda)[:3] for i in range(4)]
    x = synth.activations(M, K, torch.bfloat16, seed=M, device=cuda)
    _run_modes(lambda: _gptq_chain(x, layers, gs), overlap_mode)


@pytest.mark.parametrize("M", [1, 8])
def test_nvfp4_decode_chain_identical_under_every_mode(cuda, overlap_mode, M):
    K = N = 2048
    layers = [synth.nvfp4_weights(K, N, seed=50 + i, device=cuda) for i in range(4)]
    x = synth.activations(M, K, torch.bfloat16, seed=M, device=cuda)
    _run_modes(lambda: _fp4_chain(x, layers), overlap_mode)


def test_dependent_mode_sees_weights_written_just_before(cuda, overlap_mode):
    overlap_mode(L.W4_OVERLAP_DEPENDENT)
    K, N, gs = 4096, 1024, 128
    w0 = synth.gptq_weights(K, N, gs, asym=True, seed=60, device=cuda)[:3]
    w1 = synth.gptq_weights(K, N, gs, asym=True, seed=61, device=cuda)[:3]
    x = synth.activations(4, K, torch.bfloat16, seed=62, device=cuda)
    want = ops.gptq_gemm(x, *w1, gs, 1)
    buf = [t.clone() for t in w0]
    for _ in range(3):
        for t, src in zip(buf, w0):
            t.copy_(src)
        ops.gptq_gemm(x, *buf, gs, 1)
        for t, src in zip(buf, w1):
            t.copy_(src)  # the kernel just before the GEMM rewrites its weights
        got = ops.gptq_gemm(x, *buf, gs, 1)
        assert torch.equal(got, want)


def test_mode_is_validated(cuda, overlap_mode):
    with pytest.raises(L.W4Error):
        overlap_mode(7)
    overlap_mode(L.W4_OVERLAP_STATIC_WEIGHTS)
    assert L.lib().w4_get_launch_overlap() == L.W4_OVERLAP_STATIC_WEIGHTS
