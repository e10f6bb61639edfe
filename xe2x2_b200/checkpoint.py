"""Checkpoint loading for the quantized linear layers.

* safetensors reader / writer (the public format: an 8-byte little-endian header
  length, a JSON header mapping each tensor name to ``dtype``, ``shape`` and
  ``data_offsets`` [begin, end) into the data section that follows, and an
  optional ``__metadata__`` entry).  The reference reads GPTQ checkpoints the
  same way for I32 / F16 tensors (kernels/nvfp4/gptq_s4_dump.py:32-58); this
  reader also takes BF16, F32, U8, I8, I64 and F8_E4M3, sharded checkpoints
  (``model.safetensors.index.json``) and validates every header entry.
* GPTQ layers: ``<prefix>.qweight`` i32 [K/8, N], ``.qzeros`` i32 [K/gs, N/8],
  ``.scales`` f16 [K/gs, N], ``.g_idx`` i32 [K] (optional), with the
  quantisation settings of ``quantize_config.json`` or ``config.json``'s
  ``quantization_config`` (reference: gptq_s4_dump.py:95-114 walks the
  ``.qweight`` prefixes, unpacks the nibbles and checks g_idx linearity).
* NVFP4 layers in the ModelOpt layout described by ``hf_quant_config.json``:
  ``<prefix>.weight`` u8 [N, K/2] (two E2M1 codes per byte, low nibble = even
  k), ``.weight_scale`` e4m3 [N, K/16], ``.weight_scale_2`` f32 (the tensor
  scale), ``.input_scale`` f32 (the activation tensor scale).  Only group 16 is
  NVFP4: a group-32 entry is a different format (the reference's
  kernels/nvfp4/g16_scale_landmine.py:20-48 counts g16 / g32 layers and shows
  that one scale per 32 k cannot reproduce two g16 scales), so it is rejected.

Host-side only: tensors are read on the CPU and moved to the device once.
"""
from __future__ import annotations

import json
import math
import os
import struct
from dataclasses import dataclass
from typing import Dict, Optional

import numpy as np
import torch


class CheckpointError(ValueError):
    """A malformed or unsupported checkpoint (the message names the file / tensor)."""


# safetensors dtype -> (numpy storage dtype, torch dtype)
_DTYPES = {
    "BOOL": (np.bool_, torch.bool),
    "U8": (np.uint8, torch.uint8),
    "I8": (np.int8, torch.int8),
    "I16": (np.dtype("<i2"), torch.int16),
    "I32": (np.dtype("<i4"), torch.int32),
    "I64": (np.dtype("<i8"), torch.int64),
    "F16": (np.dtype("<f2"), torch.float16),
    "BF16": (np.dtype("<u2"), torch.bfloat16),  # stored as raw 16-bit patterns
    "F32": (np.dtype("<f4"), torch.float32),
    "F64": (np.dtype("<f8"), torch.float64),
    "F8_E4M3": (np.uint8, torch.float8_e4m3fn),  # raw bytes
}
_TORCH_TO_ST = {t: k for k, (_, t) in _DTYPES.items()}
_MAX_HEADER = 100 * 2**20


class SafeTensors:
    """One ``.safetensors`` file, header parsed and checked; tensors are read lazily."""

    def __init__(self, path: str):
        self.path = path
        size = os.path.getsize(path)
        with open(path, "rb") as f:
            head = f.read(8)
            if len(head) != 8:
                raise CheckpointError(f"{path}: shorter than the 8-byte header length")
            (hlen,) = struct.unpack("<Q", head)
            if hlen > min(_MAX_HEADER, size - 8):
                raise CheckpointError(f"{path}: header length {hlen} exceeds the file ({size} bytes)")
            try:
                header = json.loads(f.read(hlen))
            except (UnicodeDecodeError, json.JSONDecodeError) as e:
                raise CheckpointError(f"{path}: header is not JSON ({e})") from None
        if not isinstance(header, dict):
            raise CheckpointError(f"{path}: header is not a JSON object")
        self.data_start = 8 + hlen
        data_len = size - self.data_start
        self.metadata = header.pop("__metadata__", None) or {}
        self._info = {}
        for name, info in header.items():
            if not isinstance(info, dict) or not {"dtype", "shape", "data_offsets"} <= set(info):
                raise CheckpointError(f"{path}: entry {name!r} lacks dtype / shape / data_offsets")
            dt = info["dtype"]
            if dt not in _DTYPES:
                raise CheckpointError(f"{path}: {name}: unsupported dtype {dt!r}")
            shape = info["shape"]
            if not isinstance(shape, list) or not all(isinstance(d, int) and d >= 0 for d in shape):
                raise CheckpointError(f"{path}: {name}: bad shape {shape!r}")
            offs = info["data_offsets"]
            if not (isinstance(offs, list) and len(offs) == 2 and all(isinstance(o, int) for o in offs)):
                raise CheckpointError(f"{path}: {name}: bad data_offsets {offs!r}")
            b, e = offs
            nbytes = math.prod(shape) * np.dtype(_DTYPES[dt][0]).itemsize
            if not (0 <= b <= e <= data_len) or e - b != nbytes:
                raise CheckpointError(f"{path}: {name}: data_offsets {b}..{e} do not hold "
                                      f"{nbytes} bytes inside a {data_len}-byte data section")
            self._info[name] = (dt, tuple(shape), b, e)

    def names(self) -> list:
        return sorted(self._info)

    def __contains__(self, name: str) -> bool:
        return name in self._info

    def dtype(self, name: str) -> str:
        return self._entry(name)[0]

    def shape(self, name: str) -> tuple:
        return self._entry(name)[1]

    def _entry(self, name):
        try:
            return self._info[name]
        except KeyError:
            raise CheckpointError(f"{self.path}: no tensor {name!r}") from None

    def numpy(self, name: str) -> np.ndarray:
        """The stored values (BF16 as uint16 patterns, F8_E4M3 as bytes), read-only."""
        dt, shape, b, e = self._entry(name)
        npdt = np.dtype(_DTYPES[dt][0])
        if e == b:
            return np.empty(shape, dtype=npdt)
        mm = np.memmap(self.path, dtype=np.uint8, mode="r", offset=self.data_start + b, shape=(e - b,))
        return mm.view(npdt).reshape(shape)

    def tensor(self, name: str, device=None) -> torch.Tensor:
        dt = self.dtype(name)
        t = torch.from_numpy(np.array(self.numpy(name)))  # a private, writable copy
        if dt in ("BF16", "F8_E4M3"):
            t = t.view(_DTYPES[dt][1])
        return t if device is None else t.to(device)


class Checkpoint:
    """A checkpoint directory, a single ``.safetensors`` file, or a sharded set
    indexed by ``model.safetensors.index.json`` (``weight_map``: name -> file)."""

    def __init__(self, path: str):
        self.root = path if os.path.isdir(path) else os.path.dirname(os.path.abspath(path))
        files = {}
        if os.path.isfile(path):
            files[path] = SafeTensors(path)
        else:
            index = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(index):
                with open(index) as f:
                    wm = json.load(f).get("weight_map") or {}
                for fn in sorted(set(wm.values())):
                    p = os.path.join(path, fn)
                    files[p] = SafeTensors(p)
            else:
                for fn in sorted(os.listdir(path)):
                    if fn.endswith(".safetensors"):
                        p = os.path.join(path, fn)
                        files[p] = SafeTensors(p)
        if not files:
            raise CheckpointError(f"{path}: no .safetensors files")
        self._where: Dict[str, SafeTensors] = {}
        for st in files.values():
            for n in st.names():
                if n in self._where:
                    raise CheckpointError(f"{n} is stored in both {self._where[n].path} and {st.path}")
                self._where[n] = st

    def names(self) -> list:
        return sorted(self._where)

    def __contains__(self, name: str) -> bool:
        return name in self._where

    def file_of(self, name: str) -> SafeTensors:
        try:
            return self._where[name]
        except KeyError:
            raise CheckpointError(f"checkpoint has no tensor {name!r}") from None

    def shape(self, name: str) -> tuple:
        return self.file_of(name).shape(name)

    def dtype(self, name: str) -> str:
        return self.file_of(name).dtype(name)

    def numpy(self, name: str) -> np.ndarray:
        return self.file_of(name).numpy(name)

    def tensor(self, name: str, device=None) -> torch.Tensor:
        return self.file_of(name).tensor(name, device)

    def json(self, filename: str) -> Optional[dict]:
        p = os.path.join(self.root, filename)
        if not os.path.exists(p):
            return None
        with open(p) as f:
            return json.load(f)


def save_safetensors(path: str, tensors: Dict[str, object], metadata: Optional[Dict[str, str]] = None) -> None:
    """Write numpy arrays / CPU torch tensors as one ``.safetensors`` file (names sorted,
    data packed in that order, header padded with spaces to a multiple of 8 bytes)."""
    entries, blobs, off = {}, [], 0
    for name in sorted(tensors):
        v = tensors[name]
        if isinstance(v, torch.Tensor):
            v = v.detach().cpu().contiguous()
            if v.dtype not in _TORCH_TO_ST:
                raise CheckpointError(f"{name}: dtype {v.dtype} has no safetensors code")
            dt = _TORCH_TO_ST[v.dtype]
            raw = v.reshape(-1).view(torch.uint8).numpy().tobytes() if v.numel() else b""
            shape = list(v.shape)
        else:
            a = np.ascontiguousarray(v)
            dt = next((k for k, (npdt, _) in _DTYPES.items()
                       if k not in ("BF16", "F8_E4M3") and np.dtype(npdt) == a.dtype.newbyteorder("<")), None)
            if dt is None:
                raise CheckpointError(f"{name}: numpy dtype {a.dtype} has no safetensors code")
            raw = a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes()
            shape = list(a.shape)
        entries[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        entries["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    head = json.dumps(entries, separators=(",", ":")).encode()
    head += b" " * (-len(head) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(head)))
        f.write(head)
        for b in blobs:
            f.write(b)


# ===================================================================== GPTQ
@dataclass
class GPTQConfig:
    bits: int = 4
    group_size: int = 128  # -1 in a config means one group over all of K
    desc_act: bool = False
    sym: bool = True
    zero_offset: int = 1  # stored zero + 1 ("gptq"); 0 for "gptq_v2"


def gptq_config(src) -> GPTQConfig:
    """GPTQConfig from a Checkpoint (quantize_config.json, else config.json's
    quantization_config) or from such a dict."""
    if isinstance(src, Checkpoint):
        d = src.json("quantize_config.json")
        if d is None:
            d = (src.json("config.json") or {}).get("quantization_config")
        if d is None:
            raise CheckpointError(f"{src.root}: no quantize_config.json or config.json quantization_config")
    else:
        d = dict(src)
    method = str(d.get("quant_method", "gptq")).lower()
    if method != "gptq":
        raise CheckpointError(f"quant_method {method!r} is not GPTQ")
    bits = int(d.get("bits", 4))
    if bits != 4:
        raise CheckpointError(f"GPTQ bits={bits}: only 4-bit weights are supported")
    fmt = str(d.get("checkpoint_format", "gptq")).lower()
    if fmt not in ("gptq", "gptq_v2"):
        raise CheckpointError(f"GPTQ checkpoint_format {fmt!r} is not gptq / gptq_v2")
    return GPTQConfig(bits=bits, group_size=int(d.get("group_size", 128)), desc_act=bool(d.get("desc_act", False)),
                      sym=bool(d.get("sym", True)), zero_offset=0 if fmt == "gptq_v2" else 1)


def gptq_prefixes(ckpt: Checkpoint) -> list:
    """Every layer prefix that has a ``.qweight`` tensor, sorted."""
    return sorted(n[: -len(".qweight")] for n in ckpt.names() if n.endswith(".qweight"))


@dataclass
class GPTQTensors:
    qweight: torch.Tensor  # i32 [K/8, N]
    qzeros: Optional[torch.Tensor]  # i32 [K/gs, N/8]; None = symmetric (zero 8)
    scales: torch.Tensor  # f16 [K/gs, N]
    g_idx: Optional[torch.Tensor]  # i32 [K]; None = k / group_size
    group_size: int
    zero_offset: int

    @property
    def K(self) -> int:
        return self.qweight.shape[0] * 8

    @property
    def N(self) -> int:
        return self.qweight.shape[1]


def load_gptq_tensors(ckpt: Checkpoint, prefix: str, cfg: Optional[GPTQConfig] = None,
                      device=None) -> GPTQTensors:
    """Read and check one GPTQ layer.  The group size comes from the shapes (K / scale
    rows) and must agree with ``cfg`` when given (without ``cfg``: GPTQ v1 zeros).  A g_idx equal to k // group_size is
    dropped (no permutation needed); qzeros whose every stored value gives zero 8 are
    dropped (the symmetric kernels)."""
    zero_offset = cfg.zero_offset if cfg is not None else 1
    need = [prefix + s for s in (".qweight", ".scales")]
    for n in need:
        if n not in ckpt:
            raise CheckpointError(f"{prefix}: missing {n}")
    for n, dt in ((prefix + ".qweight", "I32"), (prefix + ".scales", "F16"), (prefix + ".qzeros", "I32"),
                  (prefix + ".g_idx", "I32")):
        if n in ckpt and ckpt.dtype(n) != dt:
            raise CheckpointError(f"{n}: dtype {ckpt.dtype(n)}, expected {dt}")
    qw_shape, sc_shape = ckpt.shape(prefix + ".qweight"), ckpt.shape(prefix + ".scales")
    if len(qw_shape) != 2 or len(sc_shape) != 2 or sc_shape[1] != qw_shape[1]:
        raise CheckpointError(f"{prefix}: qweight {qw_shape} / scales {sc_shape} are not [K/8, N] / [G, N]")
    K, N = qw_shape[0] * 8, qw_shape[1]
    G = sc_shape[0]
    if G == 0 or K % G:
        raise CheckpointError(f"{prefix}: K={K} is not a multiple of the {G} scale rows")
    gs = K // G
    if cfg is not None and (G != 1 if cfg.group_size == -1 else gs != cfg.group_size):
        raise CheckpointError(f"{prefix}: shapes give group size {gs}, the config says {cfg.group_size}")
    qz = None
    if prefix + ".qzeros" in ckpt:
        zs = ckpt.shape(prefix + ".qzeros")
        if zs != (G, N // 8) or N % 8:
            raise CheckpointError(f"{prefix}: qzeros {zs}, expected {(G, N // 8)}")
        qz_np = ckpt.numpy(prefix + ".qzeros")
        sym_word = np.uint32(sum((8 - zero_offset) << (4 * i) for i in range(8))).view(np.int32)
        if not np.all(qz_np == sym_word):
            qz = torch.from_numpy(np.array(qz_np))
    gi = None
    if prefix + ".g_idx" in ckpt:
        if ckpt.shape(prefix + ".g_idx") != (K,):
            raise CheckpointError(f"{prefix}: g_idx {ckpt.shape(prefix + '.g_idx')}, expected ({K},)")
        gi_np = ckpt.numpy(prefix + ".g_idx")
        if gi_np.min(initial=0) < 0 or gi_np.max(initial=0) >= G:
            raise CheckpointError(f"{prefix}: g_idx values outside 0..{G - 1}")
        if not np.array_equal(gi_np, np.arange(K, dtype=np.int32) // gs):
            gi = torch.from_numpy(np.array(gi_np))
    t = GPTQTensors(ckpt.tensor(prefix + ".qweight"), qz, ckpt.tensor(prefix + ".scales"), gi, gs, zero_offset)
    if device is not None:
        t.qweight, t.scales = t.qweight.to(device), t.scales.to(device)
        t.qzeros = None if t.qzeros is None else t.qzeros.to(device)
        t.g_idx = None if t.g_idx is None else t.g_idx.to(device)
    return t


def load_gptq_linear(ckpt: Checkpoint, prefix: str, cfg: Optional[GPTQConfig] = None, device="cuda"):
    """An ops.GPTQLinear for one layer (act_order layers are repacked once on the device)."""
    from . import ops

    t = load_gptq_tensors(ckpt, prefix, cfg, device)
    return ops.GPTQLinear(t.qweight, t.qzeros, t.scales, t.g_idx, t.group_size, t.zero_offset)


# ===================================================================== NVFP4 (ModelOpt)
@dataclass
class NVFP4Config:
    quant_algo: str
    group_size: int
    layers: Dict[str, dict]  # per-layer overrides ({"quant_algo", "group_size"})
    exclude: tuple = ()

    def layer(self, prefix: str) -> tuple:
        """(quant_algo, group_size) of one layer: its own entry, else the global one."""
        info = self.layers.get(prefix)
        if info is not None:
            return str(info.get("quant_algo", self.quant_algo)), int(info.get("group_size", self.group_size))
        if any(prefix == e or (e.endswith("*") and prefix.startswith(e[:-1])) for e in self.exclude):
            return "NONE", 0
        return self.quant_algo, self.group_size


def nvfp4_config(src) -> NVFP4Config:
    """NVFP4Config from a Checkpoint (hf_quant_config.json) or from such a dict."""
    if isinstance(src, Checkpoint):
        d = src.json("hf_quant_config.json")
        if d is None:
            raise CheckpointError(f"{src.root}: no hf_quant_config.json")
    else:
        d = dict(src)
    q = d.get("quantization") or {}
    return NVFP4Config(quant_algo=str(q.get("quant_algo") or "MIXED_PRECISION"),
                       group_size=int(q.get("group_size") or 16),
                       layers=dict(q.get("quantized_layers") or {}),
                       exclude=tuple(q.get("exclude_modules") or ()))


@dataclass
class NVFP4Tensors:
    w: torch.Tensor  # u8 [K/2, N] view with stride(0) == 1 (memory [N, K/2], K contiguous)
    scale: torch.Tensor  # e4m3 [K/16, N]
    global_scale: torch.Tensor  # f32 [1]
    input_scale: Optional[torch.Tensor]  # f32 [1]: activation tensor scale, or None

    @property
    def K(self) -> int:
        return self.w.shape[0] * 2

    @property
    def N(self) -> int:
        return self.w.shape[1]


def load_nvfp4_tensors(ckpt: Checkpoint, prefix: str, cfg: Optional[NVFP4Config] = None,
                       device=None) -> NVFP4Tensors:
    """Read and check one ModelOpt NVFP4 layer into the operator layout: the packed
    codes stay [N, K/2] in memory (exposed as the [K/2, N] view the operator takes),
    the block scales are transposed once to [K/16, N]."""
    if cfg is not None:
        algo, gs = cfg.layer(prefix)
        if algo != "NVFP4":
            raise CheckpointError(f"{prefix}: quant_algo {algo!r} is not NVFP4")
        if gs != 16:
            raise CheckpointError(f"{prefix}: NVFP4 group_size {gs}: the format scales every 16 k; a "
                                  f"{gs}-wide group cannot hold two 16-k block scales")
    for suf, dt in ((".weight", "U8"), (".weight_scale", "F8_E4M3"), (".weight_scale_2", "F32")):
        n = prefix + suf
        if n not in ckpt:
            raise CheckpointError(f"{prefix}: missing {n}")
        if ckpt.dtype(n) != dt:
            raise CheckpointError(f"{n}: dtype {ckpt.dtype(n)}, expected {dt}")
    ws, ss = ckpt.shape(prefix + ".weight"), ckpt.shape(prefix + ".weight_scale")
    if len(ws) != 2 or len(ss) != 2:
        raise CheckpointError(f"{prefix}: weight {ws} / weight_scale {ss} are not 2-D")
    N, K = ws[0], ws[1] * 2
    if ss != (N, K // 16) or K % 16:
        raise CheckpointError(f"{prefix}: weight_scale {ss}, expected {(N, K // 16)} for weight {ws}")
    for n in (prefix + ".weight_scale_2", prefix + ".input_scale"):
        if n in ckpt and math.prod(ckpt.shape(n)) != 1:
            raise CheckpointError(f"{n}: shape {ckpt.shape(n)}, expected one value")
    w_nk = ckpt.tensor(prefix + ".weight")
    scale = ckpt.tensor(prefix + ".weight_scale").t().contiguous()
    g = ckpt.tensor(prefix + ".weight_scale_2").reshape(1).float()
    a = ckpt.tensor(prefix + ".input_scale").reshape(1).float() if prefix + ".input_scale" in ckpt else None
    if device is not None:
        w_nk, scale, g = w_nk.to(device), scale.to(device), g.to(device)
        a = None if a is None else a.to(device)
    return NVFP4Tensors(w_nk.t(), scale, g, a)


def nvfp4_prefixes(ckpt: Checkpoint) -> list:
    """Every layer prefix with ``.weight`` + ``.weight_scale`` + ``.weight_scale_2``, sorted."""
    return sorted(n[: -len(".weight_scale_2")] for n in ckpt.names()
                  if n.endswith(".weight_scale_2") and n[: -len("_2")] in ckpt)


def save_nvfp4_layer(tensors: Dict[str, object], prefix: str, w_kn_view: torch.Tensor, scale_kn: torch.Tensor,
                     global_scale: torch.Tensor, input_scale: Optional[torch.Tensor] = None) -> None:
    """Add one layer in the ModelOpt layout to ``tensors`` (for save_safetensors) from the
    operator layout: w [K/2, N] view with stride(0) == 1, scale e4m3 [K/16, N]."""
    tensors[prefix + ".weight"] = w_kn_view.t().contiguous().cpu()
    tensors[prefix + ".weight_scale"] = scale_kn.t().contiguous().cpu()
    tensors[prefix + ".weight_scale_2"] = global_scale.reshape(()).float().cpu()
    if input_scale is not None:
        tensors[prefix + ".input_scale"] = input_scale.reshape(()).float().cpu()


def load_nvfp4_linear(ckpt: Checkpoint, prefix: str, cfg: Optional[NVFP4Config] = None, device="cuda",
                      act_mode=None):
    """An ops.NVFP4Linear for one layer."""
    from . import ops

    t = load_nvfp4_tensors(ckpt, prefix, cfg, device)
    return ops.NVFP4Linear(t.w, t.scale, t.global_scale, t.input_scale, act_mode)


# ===================================================================== reference tile dumps
def read_s4_dump(path: str):
    """Read a GPTQ weight tile as the reference dumps it (kernels/nvfp4/gptq_s4_dump.py:153-181
    writes, kernels/esimd_dpas/dpas_s4_gptq_sc.cpp:404-440 reads): ``u32 k, u32 n`` and the
    int8 codes s4 = u - 8 in [-8, 7], [k, n] row-major; the scaled form adds ``u32 gs``
    after n and f16 scales [k/gs, n] after the codes.
    -> (s4 int8 [k, n], scales f16 [k/gs, n] or None, gs or None)."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 8:
        raise CheckpointError(f"{path}: shorter than the 8-byte header")
    k, n = struct.unpack_from("<II", data, 0)
    scales, gs, off = None, None, 8
    if len(data) != 8 + k * n:
        if len(data) < 12:
            raise CheckpointError(f"{path}: {len(data)} bytes do not hold a {k} x {n} tile")
        (gs,) = struct.unpack_from("<I", data, 8)
        if gs == 0 or k % gs or len(data) != 12 + k * n + (k // gs) * n * 2:
            raise CheckpointError(f"{path}: {len(data)} bytes match neither the plain {k} x {n} tile nor "
                                  f"the tile with group-{gs} scales")
        off = 12
        scales = np.frombuffer(data, dtype="<f2", count=(k // gs) * n, offset=12 + k * n).reshape(k // gs, n).copy()
    s4 = np.frombuffer(data, dtype=np.int8, count=k * n, offset=off).reshape(k, n).copy()
    if s4.size and (s4.min() < -8 or s4.max() > 7):
        raise CheckpointError(f"{path}: codes outside the signed 4-bit range")
    return s4, scales, gs


def write_s4_dump(path: str, s4: np.ndarray, scales: Optional[np.ndarray] = None,
                  group_size: Optional[int] = None) -> None:
    """Write a tile in the reference's dump format (see read_s4_dump)."""
    s4 = np.ascontiguousarray(s4, dtype=np.int8)
    if s4.ndim != 2 or (s4.size and (s4.min() < -8 or s4.max() > 7)):
        raise CheckpointError("s4 must be a 2-D array of codes in [-8, 7]")
    k, n = s4.shape
    with open(path, "wb") as f:
        if scales is None:
            f.write(struct.pack("<II", k, n))
            f.write(s4.tobytes())
            return
        sc = np.ascontiguousarray(scales, dtype="<f2")
        if not group_size or k % group_size or sc.shape != (k // group_size, n):
            raise CheckpointError(f"scales {sc.shape} do not match a group-{group_size} {k} x {n} tile")
        f.write(struct.pack("<III", k, n, group_size))
        f.write(s4.tobytes())
        f.write(sc.tobytes())


def gptq_tensors_from_s4(s4: np.ndarray, scales: np.ndarray, group_size: int):
    """A dumped tile as GPTQ checkpoint tensors for w4_gptq_gemm: codes u = s4 + 8 packed
    eight per int32 along K (LSB first), stored zeros 7 (zero 8 under zero_offset 1, the
    reference's u - 8), the scales unchanged.  -> (qweight i32 [k/8, n], qzeros i32 [k/gs, n/8],
    scales f16 [k/gs, n])."""
    s4 = np.asarray(s4, dtype=np.int16)
    k, n = s4.shape
    if k % 8 or n % 8 or k % group_size:
        raise CheckpointError(f"a {k} x {n} tile cannot be packed (k % 8, n % 8, k % group_size)")
    u = (s4 + 8).astype(np.uint32).reshape(k // 8, 8, n)
    qw = np.zeros((k // 8, n), dtype=np.uint32)
    for j in range(8):
        qw |= u[:, j, :] << np.uint32(4 * j)
    qz = np.full((k // group_size, n // 8), 0x77777777, dtype=np.uint32)
    return qw.view(np.int32), qz.view(np.int32), np.ascontiguousarray(scales, dtype="<f2")
