"""Checkpoint loaders end to end on the GPU: layers written as safetensors (GPTQ
act_order with its config, ModelOpt NVFP4 with hf_quant_config.json), loaded by
xe2x2_b200.checkpoint and run through the CUDA GEMMs, against the CPU oracle and
against the same tensors passed to the operators directly."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, bits16, f32, np_
from xe2x2_b200 import _lib as L
from xe2x2_b200 import checkpoint as C
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _gptq_oracle(a, t):
    return O.gptq_gemm(f32(a), np_(t.qweight), None if t.qzeros is None else np_(t.qzeros), bits16(t.scales),
                       None if t.g_idx is None else np_(t.g_idx), a.shape[0], t.N, t.K, t.group_size,
                       t.zero_offset)


@pytest.mark.parametrize("M", [1, 4, 40])
def test_golden_act_order_checkpoint_runs(cuda, M):
    ck = C.Checkpoint(os.path.join(GOLD, "gptq_tiny.safetensors"))
    (prefix,) = C.gptq_prefixes(ck)
    t = C.load_gptq_tensors(ck, prefix, device=cuda)
    assert t.g_idx is not None and t.group_size == 32
    lin = C.load_gptq_linear(ck, prefix, device=cuda)
    a = synth.activations(M, t.K, torch.bfloat16, seed=M, device=cuda)
    rf, _ = assert_gemm_close(f32(lin(a, out_dtype=torch.float32)), _gptq_oracle(a, t))
    assert rf < 4e-3


@pytest.mark.parametrize("fmt", ["gptq", "gptq_v2"])
def test_written_gptq_checkpoint_matches_direct_call(cuda, tmp_path, fmt):
    K, N, gs = 2048, 512, 128
    zo = 0 if fmt == "gptq_v2" else 1
    qw, qz, sc, gi = synth.gptq_weights(K, N, gs, asym=True, seed=5, act_order=True)
    p = "model.layers.3.mlp.down_proj"
    C.save_safetensors(str(tmp_path / "model.safetensors"),
                       {p + ".qweight": qw, p + ".qzeros": qz, p + ".scales": sc, p + ".g_idx": gi})
    (tmp_path / "quantize_config.json").write_text(json.dumps(
        {"bits": 4, "group_size": gs, "desc_act": True, "sym": False, "checkpoint_format": fmt}))
    ck = C.Checkpoint(str(tmp_path))
    lin = C.load_gptq_linear(ck, p, C.gptq_config(ck), device=cuda)
    direct = ops.GPTQLinear(qw.to(cuda), qz.to(cuda), sc.to(cuda), gi.to(cuda), gs, zo)
    for M in (1, 16, 64):
        a = synth.activations(M, K, torch.bfloat16, seed=M, device=cuda)
        assert torch.equal(lin(a), direct(a))
    t = C.load_gptq_tensors(ck, p, C.gptq_config(ck), device=cuda)
    a = synth.activations(8, K, torch.bfloat16, seed=8, device=cuda)
    assert_gemm_close(f32(lin(a, out_dtype=torch.float32)), _gptq_oracle(a, t))
    assert L.lib().w4_check_device_status() == L.W4_OK


def test_written_nvfp4_checkpoint_matches_direct_call(cuda, tmp_path):
    K, N = 1024, 512
    w, scale, gscale = synth.nvfp4_weights(K, N, seed=6)
    ins = torch.tensor([0.02])
    ts = {}
    C.save_nvfp4_layer(ts, "model.layers.0.mlp.up_proj", w, scale, gscale, ins)
    C.save_safetensors(str(tmp_path / "model.safetensors"), ts)
    (tmp_path / "hf_quant_config.json").write_text(json.dumps(
        {"quantization": {"quant_algo": "NVFP4", "group_size": 16}}))
    ck = C.Checkpoint(str(tmp_path))
    cfg = C.nvfp4_config(ck)
    lin = C.load_nvfp4_linear(ck, "model.layers.0.mlp.up_proj", cfg, device=cuda)
    wd, sd, gd = w.to(cuda), scale.to(cuda), gscale.to(cuda)
    for M in (1, 8, 64):
        x = synth.activations(M, K, torch.bfloat16, seed=M, device=cuda)
        assert torch.equal(lin(x), ops.nvfp4_gemm(x, wd, sd, gd))
    x = synth.activations(4, K, torch.bfloat16, seed=4, device=cuda)
    ref = O.nvfp4_gemm(f32(x), np_(w.contiguous()), O.NVFP4_KN, np_(scale.view(torch.uint8)), O.SCALE_E4M3,
                       float(gscale.item()), 4, N, K)
    assert_gemm_close(f32(lin(x, out_dtype=torch.float32)), ref)
    # NVFP4 activations with the layer's input_scale (block-scaled FP4 tensor cores)
    lin4 = C.load_nvfp4_linear(ck, "model.layers.0.mlp.up_proj", cfg, device=cuda, act_mode=L.W4_ACT_NVFP4)
    x = synth.activations(256, K, torch.bfloat16, seed=7, device=cuda)
    assert torch.equal(lin4(x), ops.nvfp4_gemm(x, wd, sd, gd, act_mode=L.W4_ACT_NVFP4,
                                               a_global=ins.to(cuda)))
    assert L.lib().w4_check_device_status() == L.W4_OK
