"""PyTorch-facing host API over libw4 (include/w4.h).

The names and argument meanings mirror the reference's interfaces for the
weight-only quantized linear path (hotschmoe/xe2x2):

* ``gptq_gemm_s4a(ad, bd, asd, sd, rows, cols, dk)`` -- the argument list of the
  reference kernel ``launch(q, ad, bd, asd, sd, cd, rows, cols, dk)``
  (kernels/esimd_dpas/dpas_s4_gptq_sc.cpp:146-149), returning ``cd``.
* ``nvfp4_lut_gemm_s8a(ad, pd, asd, bsd, rows, cols, dk)`` -- the reference LUT
  kernel ``launch`` (kernels/nvfp4/nibble_lut_sc.cpp:198-201).
* ``nvfp4_gemm_w4a16(x, w, bias, scale, gs)`` and
  ``nvfp4_gemm_w4a16_f8scale(x, w, bias, bscale, gscale, gs)`` -- the operator
  the reference benches call as ``torch.ops._xpu_C.*``
  (kernels/nvfp4/bench_nvfp4_m1.py:67,88); also registered as ``torch.ops.w4.*``.
* ``rmsnorm_quant_s8(x)`` -- ``launch_fused(q, x, q, s, m, k)``
  (kernels/epilogue_quant/rmsnorm_epilogue.cpp:118-119).
* ``gptq_gemm(...)`` -- the W4A16 GPTQ GEMM on checkpoint tensors
  (qweight / qzeros / scales / g_idx as read by kernels/nvfp4/gptq_s4_dump.py:106).

Every function launches on the current CUDA stream and raises ``W4Error`` on
a bad argument; there is no CPU path.
"""
from __future__ import annotations

import ctypes
import threading
import weakref

import torch

from . import _lib as L

_DT = {torch.float16: L.W4_F16, torch.bfloat16: L.W4_BF16, torch.float32: L.W4_F32,
       torch.float8_e4m3fn: L.W4_E4M3}


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("libw4 operates on CUDA tensors only (no CPU path)")


def _contig(t, name):
    if t is not None and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


class _Workspace:
    """Per-(device, stream) scratch buffer grown on demand (callers of the C ABI pass it in).

    Allocated zero-filled: every libw4 workspace starts with a sync area that must be zero
    before first use and that every call leaves zero (include/w4.h).
    """

    def __init__(self):
        self._buf = {}
        self._lock = threading.Lock()

    def get(self, dev: torch.device, nbytes: int):
        if nbytes == 0:
            return None, 0
        key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
        with self._lock:
            buf = self._buf.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
                self._buf[key] = buf
        return buf, buf.numel()


_WS = _Workspace()


# ===================================================================== GPTQ
def gptq_dequant(qweight, qzeros, scales, g_idx=None, group_size=128, zero_offset=1):
    """fp32 [K, N] = scales[g, n] * (q[k, n] - zero[g, n]), bit-exact."""
    _need_cuda(qweight, qzeros, scales, g_idx)
    K, N = qweight.shape[0] * 8, qweight.shape[1]
    out = torch.empty((K, N), dtype=torch.float32, device=qweight.device)
    L.call("w4_gptq_dequant", _p(qweight), _p(qzeros), _p(scales), _p(g_idx), K, N, group_size, zero_offset, _p(out), _stream(qweight.device))
    return out


def gptq_repack_act_order(qweight, g_idx, group_size=128):
    """Load-time act_order repack -> (qweight with groups contiguous, perm i32[K])."""
    _need_cuda(qweight, g_idx)
    K, N = qweight.shape[0] * 8, qweight.shape[1]
    out = torch.empty_like(qweight)
    perm = torch.empty(K, dtype=torch.int32, device=qweight.device)
    L.call("w4_gptq_repack_act_order", _p(qweight), _p(g_idx.to(torch.int32).contiguous()), K, N, group_size,
           _p(out), _p(perm), _stream(qweight.device))
    return out, perm


def gptq_gemm(a, qweight, qzeros, scales, group_size=128, zero_offset=1, perm=None,
              out_dtype=None, return_row_scale=False, out=None):
    """W4A16 GPTQ GEMM: a [M, K] f16/bf16 -> [M, N] (fp32 accumulate).

    ``perm`` comes from :func:`gptq_repack_act_order` (then ``qweight`` must be
    the repacked one).  ``out_dtype=torch.float8_e4m3fn`` applies the per-row
    fp8 cast and also returns the f32 row scales.  ``out`` (optional) receives
    the result in place.
    """
    _need_cuda(a, qweight, qzeros, scales, perm)
    for t, n in ((a, "a"), (qweight, "qweight"), (qzeros, "qzeros"), (scales, "scales"), (perm, "perm")):
        _contig(t, n)
    M, K = a.shape
    N = qweight.shape[1]
    if qweight.shape[0] * 8 != K:
        raise ValueError(f"qweight {tuple(qweight.shape)} does not match K={K}")
    out_dtype = out_dtype or (out.dtype if out is not None else a.dtype)
    if out is not None:
        if out.shape != (M, N) or out.dtype != out_dtype or not out.is_contiguous() or out.device != a.device:
            raise ValueError(f"out must be a contiguous {out_dtype} [{M}, {N}] tensor on {a.device}")
        c = out
    else:
        c = torch.empty((M, N), dtype=out_dtype, device=a.device)
    rs = torch.empty(M, dtype=torch.float32, device=a.device) if out_dtype == torch.float8_e4m3fn else None
    need = L.lib().w4_gptq_workspace_bytes(M, N, K, group_size, int(perm is not None), _DT[out_dtype])
    ws, wsb = _WS.get(a.device, need)
    L.call("w4_gptq_gemm", _p(a), _DT[a.dtype], _p(qweight), _p(qzeros), _p(scales), _p(perm), _p(c),
           _DT[out_dtype], _p(rs), M, N, K, group_size, zero_offset, _p(ws), wsb, _stream(a.device))
    return (c, rs) if (return_row_scale or rs is not None) else c


def gptq_gemm_s4a(ad, bd, asd, sd, rows, cols, dk):
    """The reference kernel contract: C f16 [rows, cols] from s4-packed A and B."""
    _need_cuda(ad, bd, asd, sd)
    cd = torch.empty((rows, cols), dtype=torch.float16, device=ad.device)
    L.call("w4_gptq_gemm_s4a", _p(ad), _p(bd), _p(asd), _p(sd), _p(cd), rows, cols, dk, _stream(ad.device))
    return cd


class GPTQLinear:
    """A GPTQ int4 linear layer held in HBM in checkpoint layout.

    act_order checkpoints (``g_idx`` not the identity grouping) are repacked once
    at construction; every call then gathers the activation columns by ``perm``.
    """

    def __init__(self, qweight, qzeros, scales, g_idx=None, group_size=128, zero_offset=1):
        self.group_size, self.zero_offset = group_size, zero_offset
        self.qzeros, self.scales = qzeros, scales
        self.K, self.N = qweight.shape[0] * 8, qweight.shape[1]
        self.perm = None
        if g_idx is not None:
            ident = torch.arange(self.K, device=g_idx.device, dtype=torch.int32) // group_size
            if not torch.equal(g_idx.to(torch.int32), ident):
                qweight, self.perm = gptq_repack_act_order(qweight, g_idx, group_size)
        self.qweight = qweight

    def __call__(self, a, out_dtype=None):
        return gptq_gemm(a, self.qweight, self.qzeros, self.scales, self.group_size, self.zero_offset,
                         self.perm, out_dtype)


# ===================================================================== NVFP4
def _layout_of(w, K, N):
    """[K/2, N] u8: stride(0)==1 means [N, K/2] memory (NK), contiguous means KN."""
    if w.dim() != 2 or w.shape[0] * 2 != K or w.shape[1] != N:
        raise ValueError(f"w must be u8 [K/2, N] = [{K // 2}, {N}], got {tuple(w.shape)}")
    if w.stride(0) == 1 and w.stride(1) == K // 2:
        return L.W4_NVFP4_NK
    if w.is_contiguous():
        return L.W4_NVFP4_KN
    raise ValueError("w must be [K/2, N] contiguous or its transpose view (stride(0) == 1)")


def nvfp4_dequant(w, scale, global_scale=None, K=None):
    """fp32 [K, N] = (e2m1 * block scale) * tensor scale, bit-exact.  ``w`` as in nvfp4_gemm_w4a16."""
    _need_cuda(w, scale, global_scale)
    K = K or w.shape[0] * 2
    N = w.shape[1]
    layout = _layout_of(w, K, N)
    out = torch.empty((K, N), dtype=torch.float32, device=w.device)
    sdt = L.W4_E4M3 if scale.dtype in (torch.float8_e4m3fn, torch.uint8) else L.W4_BF16
    L.call("w4_nvfp4_dequant", _p(w), layout, _p(scale), sdt, _p(global_scale), K, N, _p(out), _stream(w.device))
    return out


def nvfp4_repack_kn_to_nk(w_kn):
    """u8 [K/2, N] contiguous -> the same logical tensor stored K-contiguous (stride(0) == 1)."""
    _need_cuda(w_kn)
    K, N = w_kn.shape[0] * 2, w_kn.shape[1]
    out = torch.empty((N, K // 2), dtype=torch.uint8, device=w_kn.device)
    L.call("w4_nvfp4_repack_kn_to_nk", _p(w_kn.contiguous()), K, N, _p(out), _stream(w_kn.device))
    return out.t()


def nvfp4_quant_act(a, a_global):
    """bf16 [M, K] -> (codes u8 [M, K/2], e4m3 block scales u8 [M, K/16])."""
    _need_cuda(a, a_global)
    M, K = a.shape
    codes = torch.empty((M, K // 2), dtype=torch.uint8, device=a.device)
    sf = torch.empty((M, K // 16), dtype=torch.uint8, device=a.device)
    L.call("w4_nvfp4_quant_act", _p(_contig(a, "a")), M, K, _p(a_global), _p(codes), _p(sf), _stream(a.device))
    return codes, sf


class NVFP4Activations:
    """Activations already quantised to NVFP4 for the block-scaled GEMM: codes u8
    [rows, K/2] and UE4M3 scale atoms for rows = M rounded up to 128, with the
    tensor scale ``a_global`` they were quantised with."""

    def __init__(self, codes, sf_atoms, a_global, M, K):
        self.codes, self.sf_atoms, self.a_global, self.M, self.K = codes, sf_atoms, a_global, M, K


def rmsnorm_quant_nvfp4(x, a_global, gamma=None, eps: float = 1e-6):
    """Fused producer: RMSNorm of x (f16 / bf16 [M, K]) -> NVFP4Activations
    (y = bf16(x * inv [* gamma]) quantised as nvfp4_quant_act does)."""
    _need_cuda(x, a_global, gamma)
    M, K = x.shape
    dt = {torch.float16: L.W4_F16, torch.bfloat16: L.W4_BF16}.get(x.dtype)
    if dt is None:
        raise ValueError("x must be f16 or bf16")
    if gamma is not None and (gamma.dtype != x.dtype or gamma.shape != (K,)):
        raise ValueError(f"gamma must be {x.dtype} [{K}]")
    lib = L.lib()
    codes = torch.empty(lib.w4_nvfp4_act_codes_bytes(M, K), dtype=torch.uint8, device=x.device)
    atoms = torch.empty(lib.w4_nvfp4_scale_atoms_bytes(M, K), dtype=torch.uint8, device=x.device)
    if codes.numel() == 0:
        raise ValueError(f"K={K} must be a positive multiple of 64")
    L.call("w4_rmsnorm_quant_nvfp4", _p(_contig(x, "x")), dt, None if gamma is None else _p(_contig(gamma, "gamma")),
           float(eps), _p(a_global), _p(codes), _p(atoms), M, K, _stream(x.device))
    return NVFP4Activations(codes.view(-1, K // 2), atoms, a_global, M, K)


def nvfp4_gemm_q(act, w, scale, global_scale, out_dtype=torch.bfloat16):
    """The block-scaled NVFP4 GEMM on NVFP4Activations (see rmsnorm_quant_nvfp4)."""
    _need_cuda(act.codes, w, scale, global_scale)
    M, K, N = act.M, act.K, w.shape[1]
    layout = _layout_of(w, K, N)
    if layout != L.W4_NVFP4_NK:
        raise ValueError("w must be the [K/2, N] view of [N, K/2] memory (stride(0) == 1)")
    if scale.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise ValueError("NVFP4 activations need E4M3 weight block scales")
    atoms = _scale_atoms(scale)
    cdt = {torch.float16: L.W4_F16, torch.bfloat16: L.W4_BF16, torch.float32: L.W4_F32,
           torch.float8_e4m3fn: L.W4_E4M3}[out_dtype]
    c = torch.empty((M, N), dtype=out_dtype, device=w.device)
    rs = torch.empty(M, dtype=torch.float32, device=w.device) if cdt == L.W4_E4M3 else None
    lib = L.lib()
    need = lib.w4_nvfp4_gemm_q_workspace_bytes(M, N, K, L.W4_E4M3_ATOMS, cdt)
    ws, wsb = _WS.get(w.device, need)
    L.call("w4_nvfp4_gemm_q", _p(act.codes), _p(act.sf_atoms), _p(act.a_global), _p(w), L.W4_NVFP4_NK,
           _p(atoms), L.W4_E4M3_ATOMS, _p(global_scale), _p(c), cdt, None if rs is None else _p(rs), M, N, K,
           None if ws is None else _p(ws), wsb, _stream(w.device))
    return (c, rs) if rs is not None else c


# id(scale tensor) -> (weak reference, tensor version, rearranged atoms); an entry
# goes away with its tensor (tensors compare elementwise, so they cannot be
# dictionary keys themselves).
_SCALE_ATOMS = {}


def nvfp4_repack_scales(scale):
    """E4M3 block scales [K/16, N] -> the atom layout of the block-scaled GEMM (u8, flat)."""
    _need_cuda(scale)
    _contig(scale, "scale")
    K, N = scale.shape[0] * 16, scale.shape[1]
    nbytes = L.lib().w4_nvfp4_scale_atoms_bytes(N, K)
    atoms = torch.empty(nbytes, dtype=torch.uint8, device=scale.device)
    L.call("w4_nvfp4_repack_scales", _p(scale), K, N, _p(atoms), _stream(scale.device))
    return atoms


def _scale_atoms(scale):
    """Rearranged scales for this tensor, made once and reused while the tensor is unchanged."""
    hit = _SCALE_ATOMS.get(id(scale))
    if hit is not None and hit[0]() is scale and hit[1] == scale._version:
        return hit[2]
    atoms = nvfp4_repack_scales(scale)
    key = id(scale)
    _SCALE_ATOMS[key] = (weakref.ref(scale), scale._version, atoms)
    weakref.finalize(scale, _SCALE_ATOMS.pop, key, None)
    return atoms


def scale_atoms_cached(scale) -> bool:
    hit = _SCALE_ATOMS.get(id(scale))
    return hit is not None and hit[0]() is scale and hit[1] == scale._version


def nvfp4_gemm(x, w, scale, global_scale=None, out_dtype=torch.bfloat16, act_mode=L.W4_ACT_W4A16,
               a_global=None):
    _need_cuda(x, w, scale, global_scale, a_global)
    M, K = x.shape
    N = w.shape[1]
    layout = _layout_of(w, K, N)
    if layout == L.W4_NVFP4_KN:
        w = nvfp4_repack_kn_to_nk(w)
        layout = L.W4_NVFP4_NK
    sdt = L.W4_E4M3 if scale.dtype in (torch.float8_e4m3fn, torch.uint8) else L.W4_BF16
    if act_mode == L.W4_ACT_NVFP4 and sdt == L.W4_E4M3 and K % 64 == 0:
        scale, sdt = _scale_atoms(scale), L.W4_E4M3_ATOMS
    c = torch.empty((M, N), dtype=out_dtype, device=x.device)
    rs = torch.empty(M, dtype=torch.float32, device=x.device) if out_dtype == torch.float8_e4m3fn else None
    need = L.lib().w4_nvfp4_workspace_bytes(M, N, K, act_mode, _DT[out_dtype])
    ws, wsb = _WS.get(x.device, need)
    L.call("w4_nvfp4_gemm", _p(_contig(x, "x")), _p(w), layout, _p(_contig(scale, "scale")), sdt,
           _p(global_scale), act_mode, _p(a_global), _p(c), _DT[out_dtype], _p(rs), M, N, K, _p(ws), wsb,
           _stream(x.device))
    return (c, rs) if rs is not None else c


class NVFP4Linear:
    """An NVFP4 linear layer held in HBM: codes u8 [K/2, N] (the [N, K/2] K-contiguous
    memory of a ModelOpt checkpoint seen through its transpose), E4M3 block scales
    [K/16, N], tensor scale f32 [1] and, optionally, the activation tensor scale
    ``input_scale``.  ``act_mode`` W4A16 keeps activations in bf16; W4_ACT_NVFP4
    quantises them with ``input_scale`` and runs the block-scaled FP4 tensor-core GEMM
    (needs ``input_scale``)."""

    def __init__(self, w, scale, global_scale, input_scale=None, act_mode=None):
        self.w, self.scale, self.global_scale, self.input_scale = w, scale, global_scale, input_scale
        self.K, self.N = w.shape[0] * 2, w.shape[1]
        self.act_mode = L.W4_ACT_W4A16 if act_mode is None else act_mode
        if self.act_mode == L.W4_ACT_NVFP4 and input_scale is None:
            raise ValueError("NVFP4 activations need the layer's input_scale")

    def __call__(self, x, out_dtype=torch.bfloat16):
        if self.act_mode == L.W4_ACT_NVFP4:
            return nvfp4_gemm(x, self.w, self.scale, self.global_scale, out_dtype, L.W4_ACT_NVFP4,
                              self.input_scale)
        return nvfp4_gemm(x, self.w, self.scale, self.global_scale, out_dtype)


def nvfp4_gemm_w4a16(x, w, bias, scale, gs):
    """Reference operator signature: x bf16 [M,K], w u8 [K/2,N] (stride(0)==1), scale bf16 [K/16,N]."""
    if gs != 16:
        raise ValueError("NVFP4 block size is 16")
    out = nvfp4_gemm(x, w, scale, None)
    return out if bias is None else out + bias


def nvfp4_gemm_w4a16_f8scale(x, w, bias, bscale, gscale, gs):
    """Reference operator signature with e4m3 block scales [K/16, N] and an fp32[1] tensor scale."""
    if gs != 16:
        raise ValueError("NVFP4 block size is 16")
    out = nvfp4_gemm(x, w, bscale, gscale)
    return out if bias is None else out + bias


def nvfp4_lut_gemm_s8a(ad, pd, asd, bsd, rows, cols, dk):
    """The reference LUT kernel contract: C f16 [rows, cols] = (A_s8 . 2*e2m1) * a_s * b_s."""
    _need_cuda(ad, pd, asd, bsd)
    cd = torch.empty((rows, cols), dtype=torch.float16, device=ad.device)
    L.call("w4_nvfp4_lut_gemm_s8a", _p(ad), _p(pd), _p(asd), _p(bsd), _p(cd), rows, cols, dk, _stream(ad.device))
    return cd


# ===================================================================== epilogue quant
def rmsnorm_quant_s8(x, eps: float = 1e-6):
    """Fused RMSNorm (gamma=1) + per-row s8: x f16 [M, K] -> (q s8 [M, K], scale f32 [M])."""
    _need_cuda(x)
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    L.call("w4_rmsnorm_quant_s8", _p(_contig(x, "x")), _p(q), _p(s), M, K, eps, _stream(x.device))
    return q, s


def rowscale_fp8(y):
    """Per-row fp8-E4M3 cast: y [M, N] -> (q e4m3 [M, N], scale f32 [M])."""
    _need_cuda(y)
    M, N = y.shape
    q = torch.empty((M, N), dtype=torch.float8_e4m3fn, device=y.device)
    s = torch.empty(M, dtype=torch.float32, device=y.device)
    L.call("w4_rowscale_fp8", _p(_contig(y, "y")), _DT[y.dtype], _p(q), _p(s), M, N, _stream(y.device))
    return q, s


# ===================================================================== torch.ops.w4
_registered = False


# ===================================================================== grouped (MoE)
def _offsets(offsets, E):
    off = [int(x) for x in (offsets.tolist() if torch.is_tensor(offsets) else offsets)]
    if len(off) != E + 1:
        raise ValueError(f"offsets must hold num_experts + 1 = {E + 1} entries, got {len(off)}")
    return (ctypes.c_int32 * len(off))(*off), off[-1]


def gptq_gemm_grouped(a, qweight, qzeros, scales, offsets, group_size=128, zero_offset=1, out_dtype=None):
    """Grouped (MoE) GPTQ GEMM in one launch: expert e multiplies rows [offsets[e], offsets[e+1])
    of ``a`` (tokens sorted by expert) by its slice of the stacked weights qweight [E, K/8, N],
    qzeros [E, K/gs, N/8] or None, scales [E, K/gs, N].  ``offsets``: E + 1 host ints from 0.
    Returns [rows, N] (and the row scales for an fp8 output)."""
    _need_cuda(a, qweight, qzeros, scales)
    for t, n in ((a, "a"), (qweight, "qweight"), (qzeros, "qzeros"), (scales, "scales")):
        _contig(t, n)
    E, K8, N = qweight.shape
    K = K8 * 8
    off, rows = _offsets(offsets, E)
    if a.shape != (rows, K):
        raise ValueError(f"a must be [{rows}, {K}], got {tuple(a.shape)}")
    out_dtype = out_dtype or a.dtype
    c = torch.empty((rows, N), dtype=out_dtype, device=a.device)
    rs = torch.empty(rows, dtype=torch.float32, device=a.device) if out_dtype == torch.float8_e4m3fn else None
    need = L.lib().w4_gptq_gemm_grouped_workspace_bytes(off, E, N, K, group_size, _DT[out_dtype])
    ws, wsb = _WS.get(a.device, need)
    L.call("w4_gptq_gemm_grouped", _p(a), _DT[a.dtype], _p(qweight), _p(qzeros), _p(scales), off, E, _p(c),
           _DT[out_dtype], _p(rs), N, K, group_size, zero_offset, _p(ws), wsb, _stream(a.device))
    return (c, rs) if rs is not None else c


def nvfp4_gemm_grouped(x, w_nk, scale, global_scale, offsets, out_dtype=torch.bfloat16):
    """Grouped (MoE) NVFP4 W4A16 GEMM in one launch: w_nk u8 [E, N, K/2] (K-contiguous codes),
    E4M3 block scales [E, K/16, N], tensor scales f32 [E]; bf16 activations sorted by expert."""
    _need_cuda(x, w_nk, scale, global_scale)
    for t, n in ((x, "x"), (w_nk, "w_nk"), (scale, "scale"), (global_scale, "global_scale")):
        _contig(t, n)
    E, N, K2 = w_nk.shape
    K = K2 * 2
    off, rows = _offsets(offsets, E)
    if x.shape != (rows, K) or x.dtype != torch.bfloat16:
        raise ValueError(f"x must be bf16 [{rows}, {K}]")
    c = torch.empty((rows, N), dtype=out_dtype, device=x.device)
    rs = torch.empty(rows, dtype=torch.float32, device=x.device) if out_dtype == torch.float8_e4m3fn else None
    need = L.lib().w4_nvfp4_gemm_grouped_workspace_bytes(off, E, N, K, _DT[out_dtype])
    ws, wsb = _WS.get(x.device, need)
    L.call("w4_nvfp4_gemm_grouped", _p(x), _p(w_nk), _p(scale), _p(global_scale), off, E, _p(c), _DT[out_dtype],
           _p(rs), N, K, _p(ws), wsb, _stream(x.device))
    return (c, rs) if rs is not None else c


def register_torch_ops():
    """Expose the reference operator names as ``torch.ops.w4.*`` (CUDA only)."""
    global _registered
    if _registered:
        return
    lib = torch.library.Library("w4", "DEF")
    lib.define("nvfp4_gemm_w4a16(Tensor x, Tensor w, Tensor? bias, Tensor scale, int gs) -> Tensor")
    lib.define("nvfp4_gemm_w4a16_f8scale(Tensor x, Tensor w, Tensor? bias, Tensor bscale, Tensor gscale, "
               "int gs) -> Tensor")
    lib.define("gptq_gemm(Tensor a, Tensor qweight, Tensor? qzeros, Tensor scales, Tensor? perm, "
               "int group_size, int zero_offset) -> Tensor")
    lib.impl("nvfp4_gemm_w4a16", nvfp4_gemm_w4a16, "CUDA")
    lib.impl("nvfp4_gemm_w4a16_f8scale", nvfp4_gemm_w4a16_f8scale, "CUDA")
    lib.impl("gptq_gemm",
             lambda a, qw, qz, sc, perm, gs, zo: gptq_gemm(a, qw, qz, sc, gs, zo, perm), "CUDA")
    globals()["_torch_lib"] = lib
    _registered = True
