"""Checkpoint loaders (CPU): the safetensors reader against the reference's own
reader (golden fixture), header validation, sharded checkpoints, GPTQ and
ModelOpt-NVFP4 layer loading and their configuration files."""
import json
import os
import struct

import numpy as np
import pytest
import torch

from xe2x2_b200 import checkpoint as C

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


def test_reader_matches_reference_reader_on_golden_file():
    """gptq_tiny.safetensors read by kernels/nvfp4/gptq_s4_dump.py:32-58 (recorded in
    gptq_tiny_ref.npz) and by this reader give identical arrays."""
    ref = np.load(os.path.join(GOLD, "gptq_tiny_ref.npz"))
    st = C.SafeTensors(os.path.join(GOLD, "gptq_tiny.safetensors"))
    assert st.names() == sorted(ref.files)
    for n in ref.files:
        got = st.numpy(n)
        assert got.dtype == ref[n].dtype and got.shape == ref[n].shape, n
        assert np.array_equal(got, ref[n]), n
    assert st.metadata == {"format": "pt"}


def test_writer_is_deterministic_against_golden_file(tmp_path):
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    p = tmp_path / "again.safetensors"
    mg.write_tiny_checkpoint(str(p))
    with open(p, "rb") as a, open(os.path.join(GOLD, "gptq_tiny.safetensors"), "rb") as b:
        assert a.read() == b.read()


def test_round_trip_every_dtype(tmp_path):
    g = torch.Generator().manual_seed(0)
    ts = {
        "a.bf16": torch.randn(3, 5, generator=g).to(torch.bfloat16),
        "a.f16": torch.randn(4, generator=g).half(),
        "a.f32": torch.randn(2, 2, 2, generator=g),
        "a.f8": torch.randn(6, 4, generator=g).to(torch.float8_e4m3fn),
        "b.u8": torch.randint(0, 256, (7,), generator=g, dtype=torch.uint8),
        "b.i8": torch.randint(-128, 128, (3, 3), generator=g, dtype=torch.int8),
        "b.i32": torch.randint(-2**31, 2**31 - 1, (5, 2), generator=g, dtype=torch.int32),
        "b.i64": torch.arange(4, dtype=torch.int64) - 2,
        "c.scalar": torch.tensor(0.125),
        "c.empty": torch.empty(0, 4),
        "c.np": np.arange(6, dtype=np.int16).reshape(2, 3),
    }
    p = tmp_path / "x.safetensors"
    C.save_safetensors(str(p), ts, metadata={"k": 1})
    st = C.SafeTensors(str(p))
    assert st.metadata == {"k": "1"}
    assert st.names() == sorted(ts)
    for n, v in ts.items():
        got = st.tensor(n)
        want = torch.from_numpy(v) if isinstance(v, np.ndarray) else v
        assert got.dtype == want.dtype and got.shape == want.shape, n
        assert torch.equal(got.view(torch.uint8) if got.is_floating_point() and got.numel() and got.dim() else got,
                           want.view(torch.uint8) if want.is_floating_point() and want.numel() and want.dim()
                           else want), n
    with open(p, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
    assert hlen % 8 == 0


def _raw(tmp_path, header: bytes, data: bytes = b"", hlen=None):
    p = tmp_path / "bad.safetensors"
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(header) if hlen is None else hlen))
        f.write(header)
        f.write(data)
    return str(p)


@pytest.mark.parametrize("header,data,hlen,msg", [
    (b"{}", b"", 10**9, "exceeds"),
    (b"{not json", b"", None, "not JSON"),
    (b"[1, 2]", b"", None, "not a JSON object"),
    (b'{"t": {"dtype": "I32", "shape": [2]}}', b"", None, "lacks"),
    (b'{"t": {"dtype": "Q4", "shape": [2], "data_offsets": [0, 8]}}', b"\0" * 8, None, "unsupported dtype"),
    (b'{"t": {"dtype": "I32", "shape": [-2], "data_offsets": [0, 8]}}', b"\0" * 8, None, "bad shape"),
    (b'{"t": {"dtype": "I32", "shape": [2], "data_offsets": [0, 12]}}', b"\0" * 8, None, "do not hold"),
    (b'{"t": {"dtype": "I32", "shape": [3], "data_offsets": [0, 8]}}', b"\0" * 8, None, "do not hold"),
    (b'{"t": {"dtype": "I32", "shape": [2], "data_offsets": [0]}}', b"\0" * 8, None, "bad data_offsets"),
])
def test_header_validation(tmp_path, header, data, hlen, msg):
    with pytest.raises(C.CheckpointError, match=msg):
        C.SafeTensors(_raw(tmp_path, header, data, hlen))


def test_truncated_file(tmp_path):
    p = tmp_path / "t.safetensors"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(C.CheckpointError, match="shorter"):
        C.SafeTensors(str(p))


def test_sharded_checkpoint_and_duplicates(tmp_path):
    C.save_safetensors(str(tmp_path / "m-1.safetensors"), {"x.a": np.ones(3, np.int32)})
    C.save_safetensors(str(tmp_path / "m-2.safetensors"), {"x.b": np.zeros(2, np.float32)})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {"x.a": "m-1.safetensors", "x.b": "m-2.safetensors"}}))
    ck = C.Checkpoint(str(tmp_path))
    assert ck.names() == ["x.a", "x.b"]
    assert ck.file_of("x.b").path.endswith("m-2.safetensors")
    assert ck.tensor("x.a").tolist() == [1, 1, 1]
    with pytest.raises(C.CheckpointError, match="no tensor"):
        ck.tensor("x.c")
    os.remove(tmp_path / "model.safetensors.index.json")
    C.save_safetensors(str(tmp_path / "m-3.safetensors"), {"x.a": np.ones(1, np.int32)})
    with pytest.raises(C.CheckpointError, match="stored in both"):
        C.Checkpoint(str(tmp_path))


# ---------------------------------------------------------------- GPTQ
def _gptq_layer(K, N, gs, sym=False, zero_offset=1, act_order=False, seed=0):
    rng = np.random.default_rng(seed)
    qw = rng.integers(-2**31, 2**31, size=(K // 8, N), dtype=np.int64).astype(np.int32)
    if sym:
        nib = 8 - zero_offset
        word = np.uint32(sum(nib << (4 * i) for i in range(8))).view(np.int32)
        qz = np.full((K // gs, N // 8), word, dtype=np.int32)
    else:
        qz = rng.integers(-2**31, 2**31, size=(K // gs, N // 8), dtype=np.int64).astype(np.int32)
    sc = (np.abs(rng.normal(0, 0.02, size=(K // gs, N))) + 1e-3).astype(np.float16)
    gi = np.arange(K, dtype=np.int32) // gs
    if act_order:
        gi = rng.permutation(gi).astype(np.int32)
    return {"qweight": qw, "qzeros": qz, "scales": sc, "g_idx": gi}


def _write_gptq(path, layers, cfg=None, cfg_name="quantize_config.json"):
    ts = {f"{p}.{k}": v for p, d in layers.items() for k, v in d.items()}
    os.makedirs(path, exist_ok=True)
    C.save_safetensors(os.path.join(path, "model.safetensors"), ts)
    if cfg is not None:
        with open(os.path.join(path, cfg_name), "w") as f:
            json.dump(cfg if cfg_name != "config.json" else {"quantization_config": cfg}, f)


def test_gptq_layers_load_with_their_config(tmp_path):
    layers = {
        "model.layers.0.self_attn.o_proj": _gptq_layer(256, 64, 128, seed=1),
        "model.layers.0.mlp.down_proj": _gptq_layer(512, 32, 128, act_order=True, seed=2),
        "model.layers.0.mlp.up_proj": _gptq_layer(256, 96, 128, sym=True, seed=3),
    }
    _write_gptq(tmp_path, layers, {"bits": 4, "group_size": 128, "desc_act": True, "sym": False,
                                   "quant_method": "gptq"})
    ck = C.Checkpoint(str(tmp_path))
    cfg = C.gptq_config(ck)
    assert (cfg.group_size, cfg.desc_act, cfg.zero_offset) == (128, True, 1)
    assert C.gptq_prefixes(ck) == sorted(layers)
    o = C.load_gptq_tensors(ck, "model.layers.0.self_attn.o_proj", cfg)
    assert (o.K, o.N, o.group_size) == (256, 64, 128)
    assert o.g_idx is None  # identity grouping dropped
    assert np.array_equal(o.qweight.numpy(), layers["model.layers.0.self_attn.o_proj"]["qweight"])
    assert np.array_equal(o.qzeros.numpy(), layers["model.layers.0.self_attn.o_proj"]["qzeros"])
    assert o.scales.dtype == torch.float16
    d = C.load_gptq_tensors(ck, "model.layers.0.mlp.down_proj", cfg)
    assert d.g_idx is not None and np.array_equal(d.g_idx.numpy(), layers["model.layers.0.mlp.down_proj"]["g_idx"])
    u = C.load_gptq_tensors(ck, "model.layers.0.mlp.up_proj", cfg)
    assert u.qzeros is None  # every stored zero is 7 -> effective 8: the symmetric kernels


def test_gptq_config_sources_and_rejections(tmp_path):
    _write_gptq(tmp_path, {"l": _gptq_layer(128, 32, 64)},
                {"bits": 4, "group_size": 64, "checkpoint_format": "gptq_v2"}, cfg_name="config.json")
    ck = C.Checkpoint(str(tmp_path))
    cfg = C.gptq_config(ck)
    assert cfg.zero_offset == 0 and cfg.group_size == 64
    with pytest.raises(C.CheckpointError, match="only 4-bit"):
        C.gptq_config({"bits": 8})
    with pytest.raises(C.CheckpointError, match="not GPTQ"):
        C.gptq_config({"quant_method": "awq"})
    with pytest.raises(C.CheckpointError, match="group size 64, the config says 128"):
        C.load_gptq_tensors(ck, "l", C.GPTQConfig(group_size=128))


def test_gptq_shape_and_dtype_checks(tmp_path):
    lay = _gptq_layer(128, 32, 64)
    bad = dict(lay, scales=lay["scales"].astype(np.float32))
    _write_gptq(tmp_path / "a", {"l": bad})
    with pytest.raises(C.CheckpointError, match="expected F16"):
        C.load_gptq_tensors(C.Checkpoint(str(tmp_path / "a")), "l")
    bad = dict(lay, qzeros=lay["qzeros"][:, :2])
    _write_gptq(tmp_path / "b", {"l": bad})
    with pytest.raises(C.CheckpointError, match="qzeros"):
        C.load_gptq_tensors(C.Checkpoint(str(tmp_path / "b")), "l")
    bad = dict(lay, g_idx=np.full(128, 7, np.int32))
    _write_gptq(tmp_path / "c", {"l": bad})
    with pytest.raises(C.CheckpointError, match="g_idx values"):
        C.load_gptq_tensors(C.Checkpoint(str(tmp_path / "c")), "l")
    with pytest.raises(C.CheckpointError, match="missing"):
        C.load_gptq_tensors(C.Checkpoint(str(tmp_path / "c")), "nope")


# ---------------------------------------------------------------- NVFP4 (ModelOpt)
def _nvfp4_layer(K, N, seed=0):
    g = torch.Generator().manual_seed(seed)
    w_nk = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
    sc_nk = (2.0 ** torch.randint(-6, 3, (N, K // 16), generator=g).float()).to(torch.float8_e4m3fn)
    return {"weight": w_nk, "weight_scale": sc_nk, "weight_scale_2": torch.tensor(1 / 448.0),
            "input_scale": torch.tensor(0.01)}


def _write_nvfp4(path, layers, qcfg):
    os.makedirs(path, exist_ok=True)
    C.save_safetensors(os.path.join(path, "model.safetensors"),
                       {f"{p}.{k}": v for p, d in layers.items() for k, v in d.items()})
    with open(os.path.join(path, "hf_quant_config.json"), "w") as f:
        json.dump({"producer": {"name": "modelopt"}, "quantization": qcfg}, f)


def test_nvfp4_layers_load_into_operator_layout(tmp_path):
    lay = _nvfp4_layer(256, 64, seed=4)
    _write_nvfp4(tmp_path, {"model.layers.0.mlp.gate_proj": lay, "lm_head": lay},
                 {"quant_algo": "NVFP4", "group_size": 16, "exclude_modules": ["lm_head"]})
    ck = C.Checkpoint(str(tmp_path))
    cfg = C.nvfp4_config(ck)
    assert C.nvfp4_prefixes(ck) == ["lm_head", "model.layers.0.mlp.gate_proj"]
    t = C.load_nvfp4_tensors(ck, "model.layers.0.mlp.gate_proj", cfg)
    assert (t.K, t.N) == (256, 64)
    assert t.w.shape == (128, 64) and t.w.stride() == (1, 128)  # [K/2, N] view of [N, K/2] memory
    assert torch.equal(t.w.t(), lay["weight"])
    assert t.scale.shape == (16, 64) and t.scale.is_contiguous()
    assert torch.equal(t.scale.view(torch.uint8), lay["weight_scale"].t().contiguous().view(torch.uint8))
    assert t.global_scale.shape == (1,) and float(t.global_scale) == pytest.approx(1 / 448.0)
    assert float(t.input_scale) == pytest.approx(0.01)
    with pytest.raises(C.CheckpointError, match="not NVFP4"):
        C.load_nvfp4_tensors(ck, "lm_head", cfg)  # excluded: left unquantised


def test_nvfp4_per_layer_entries_and_group_size(tmp_path):
    lay = _nvfp4_layer(128, 32)
    _write_nvfp4(tmp_path, {"a": lay, "b": lay, "c": lay},
                 {"quant_algo": "MIXED_PRECISION", "quantized_layers": {
                     "a": {"quant_algo": "NVFP4", "group_size": 16},
                     "b": {"quant_algo": "NVFP4", "group_size": 32},
                     "c": {"quant_algo": "FP8"}}})
    ck = C.Checkpoint(str(tmp_path))
    cfg = C.nvfp4_config(ck)
    C.load_nvfp4_tensors(ck, "a", cfg)
    with pytest.raises(C.CheckpointError, match="group_size 32"):
        C.load_nvfp4_tensors(ck, "b", cfg)
    with pytest.raises(C.CheckpointError, match="FP8"):
        C.load_nvfp4_tensors(ck, "c", cfg)


def test_nvfp4_shape_checks(tmp_path):
    lay = _nvfp4_layer(128, 32)
    lay["weight_scale"] = lay["weight_scale"][:, :4]
    _write_nvfp4(tmp_path, {"a": lay}, {"quant_algo": "NVFP4", "group_size": 16})
    with pytest.raises(C.CheckpointError, match="weight_scale"):
        C.load_nvfp4_tensors(C.Checkpoint(str(tmp_path)), "a")


def test_save_nvfp4_layer_inverts_load(tmp_path):
    lay = _nvfp4_layer(128, 48, seed=9)
    ts = {}
    C.save_nvfp4_layer(ts, "x", lay["weight"].t(), lay["weight_scale"].t().contiguous(),
                       lay["weight_scale_2"].reshape(1), lay["input_scale"])
    C.save_safetensors(str(tmp_path / "m.safetensors"), ts)
    t = C.load_nvfp4_tensors(C.Checkpoint(str(tmp_path)), "x")
    assert torch.equal(t.w.t(), lay["weight"])


# ---------------------------------------------------------------- reference tile dumps
def test_reads_the_reference_tile_dumps():
    """gptq_tiny_s4[_sc].bin were written by the reference's own gptq_s4_dump.py main()
    from gptq_tiny.safetensors: the codes are its u - 8 and the scaled form carries its
    group-128 header and first scale row."""
    import oracle as O

    ck = C.Checkpoint(os.path.join(GOLD, "gptq_tiny.safetensors"))
    (p,) = C.gptq_prefixes(ck)
    u = O.unpack_i32_nibbles_first(ck.numpy(p + ".qweight")).astype(np.int16)
    s4, sc, gs = C.read_s4_dump(os.path.join(GOLD, "gptq_tiny_s4.bin"))
    assert sc is None and gs is None and s4.shape == (128, 64)
    assert np.array_equal(s4.astype(np.int16), u - 8)
    s4b, scb, gsb = C.read_s4_dump(os.path.join(GOLD, "gptq_tiny_s4_sc.bin"))
    assert gsb == 128 and np.array_equal(s4b, s4)
    assert np.array_equal(scb, ck.numpy(p + ".scales")[:1])


def test_writer_reproduces_the_reference_dumps(tmp_path):
    s4, _, _ = C.read_s4_dump(os.path.join(GOLD, "gptq_tiny_s4.bin"))
    _, sc, gs = C.read_s4_dump(os.path.join(GOLD, "gptq_tiny_s4_sc.bin"))
    C.write_s4_dump(str(tmp_path / "a.bin"), s4)
    C.write_s4_dump(str(tmp_path / "b.bin"), s4, sc, gs)
    for mine, ref in (("a.bin", "gptq_tiny_s4.bin"), ("b.bin", "gptq_tiny_s4_sc.bin")):
        assert (tmp_path / mine).read_bytes() == open(os.path.join(GOLD, ref), "rb").read()


def test_dump_as_gptq_tensors_dequantises_to_s4_times_scale():
    import oracle as O

    rng = np.random.default_rng(7)
    k, n, gs = 256, 32, 64
    s4 = rng.integers(-8, 8, size=(k, n)).astype(np.int8)
    sc = (np.abs(rng.normal(0, 0.02, size=(k // gs, n))) + 1e-3).astype(np.float16)
    qw, qz, sc2 = C.gptq_tensors_from_s4(s4, sc, gs)
    assert qw.dtype == np.int32 and qw.shape == (k // 8, n) and qz.shape == (k // gs, n // 8)
    w = O.gptq_dequant(qw, qz, sc2.view(np.uint16), None, k, n, gs, 1)
    want = s4.astype(np.float32) * np.repeat(sc.astype(np.float32), gs, axis=0)
    assert np.array_equal(w, want)


def test_dump_format_errors(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(struct.pack("<II", 4, 4) + b"\0" * 15)
    with pytest.raises(C.CheckpointError, match="match neither"):
        C.read_s4_dump(str(p))
    p.write_bytes(struct.pack("<II", 2, 2) + bytes([0, 1, 2, 9]))
    with pytest.raises(C.CheckpointError, match="signed 4-bit"):
        C.read_s4_dump(str(p))
    with pytest.raises(C.CheckpointError):
        C.write_s4_dump(str(p), np.full((2, 2), 9, np.int8))
    with pytest.raises(C.CheckpointError):
        C.write_s4_dump(str(p), np.zeros((4, 2), np.int8), np.zeros((3, 2), np.float16), 2)
