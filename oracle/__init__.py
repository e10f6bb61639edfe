"""CPU oracle for the weight-only quantized linear path -- TEST INFRASTRUCTURE ONLY.

This package is the checker.  It wraps ``liboracle.so`` (plain C, built from
``w4_oracle.c`` by ``oracle/Makefile``), a restatement of the host loops of the
reference lab hotschmoe/xe2x2 (each C function cites the reference file:line it
follows).  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline /
``--impl reference`` legs of ``bench.py`` may import it; the product package
``xe2x2_b200`` never does.

Parity pin: the oracle is checked against the reference's own known answers
(the E2M1-bitcast negative's max_abs 352 / 1408, the integer-exact s4 dot and
group-scale closures, the RMSNorm-s8 ``max_abs <= 1`` contract) and against the
reference's importable unpackers (``kernels/nvfp4/gptq_s4_dump.py:61-73``) through
the fixtures in ``tests/golden/``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

NVFP4_KN = 0
NVFP4_NK = 1
SCALE_E4M3 = 0
SCALE_BF16 = 1


def build(force: bool = False) -> str:
    """Compile liboracle.so with oracle/Makefile (needs gcc)."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t
_U = ctypes.c_uint


def _declare(L):
    sig = {
        "orc_f16_to_f32": (_F, [ctypes.c_uint16]),
        "orc_f32_to_f16": (ctypes.c_uint16, [_F]),
        "orc_bf16_to_f32": (_F, [ctypes.c_uint16]),
        "orc_f32_to_bf16": (ctypes.c_uint16, [_F]),
        "orc_e2m1_value": (_F, [ctypes.c_uint8]),
        "orc_e2m1_from_f32": (ctypes.c_uint8, [_F]),
        "orc_e4m3_value": (_F, [ctypes.c_uint8]),
        "orc_e4m3_from_f32": (ctypes.c_uint8, [_F]),
        "orc_e2m1_q": (ctypes.c_int8, [ctypes.c_uint8]),
        "orc_bitcast_nibble_s4": (ctypes.c_int8, [ctypes.c_uint8]),
        "orc_fill_s4": (None, [_P, _Z, _U]),
        "orc_fill_s8": (None, [_P, _Z, _U]),
        "orc_fill_nibbles": (None, [_P, _Z, _U]),
        "orc_fill_e2m1_bitcast": (None, [_P, _P, _Z, _U]),
        "orc_fill_rmsnorm_x": (None, [_P, _Z]),
        "orc_unpack_i32_nibbles_first": (None, [_P, _I, _I, _P]),
        "orc_unpack_i32_nibbles_last": (None, [_P, _I, _I, _P]),
        "orc_pack_i32_nibbles_first": (None, [_P, _I, _I, _P]),
        "orc_pack_i32_nibbles_last": (None, [_P, _I, _I, _P]),
        "orc_pack_s4_along_k": (None, [_P, _I, _I, _P]),
        "orc_pack_s4_rows": (None, [_P, _I, _I, _P]),
        "orc_s32_gemm": (None, [_P, _P, _P, _I, _I, _I]),
        "orc_gptq_s4a_gemm": (None, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
        "orc_nvfp4_lut_gemm_s8a": (None, [_P, _P, _P, _P, _I, _I, _I, _P]),
        "orc_gptq_dequant": (None, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
        "orc_gptq_gemm": (None, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I]),
        "orc_gptq_act_order_perm": (None, [_P, _I, _I, _P]),
        "orc_nvfp4_dequant": (None, [_P, _I, _P, _I, _F, _I, _I, _P]),
        "orc_nvfp4_gemm": (None, [_P, _P, _I, _P, _I, _F, _I, _I, _I, _P, _I]),
        "orc_nvfp4_quant_act": (None, [_P, _I, _I, _F, _P, _P]),
        "orc_nvfp4_act_dequant": (None, [_P, _P, _F, _I, _I, _P]),
        "orc_rmsnorm_quant_s8": (None, [_P, _P, _P, _I, _I, _F]),
        "orc_rmsnorm_nvfp4": (None, [_P, _P, _I, _I, _F, _F, _P, _P]),
        "orc_rowscale_fp8": (None, [_P, _I, _I, _P, _P]),
        "orc_cosine": (ctypes.c_double, [_P, _P, _Z]),
        "orc_max_abs": (ctypes.c_double, [_P, _P, _Z]),
        "orc_rel_frob": (ctypes.c_double, [_P, _P, _Z]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---- scalar / format helpers -------------------------------------------------
def f16_bits_to_f32(h):
    return np.ascontiguousarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def e2m1_value(nib: int) -> float:
    return lib().orc_e2m1_value(nib)


def e2m1_from_f32(x: float) -> int:
    return lib().orc_e2m1_from_f32(x)


def e4m3_value(b: int) -> float:
    return lib().orc_e4m3_value(b)


def e4m3_from_f32(x: float) -> int:
    return lib().orc_e4m3_from_f32(x)


def f32_to_bf16_bits(x: float) -> int:
    return lib().orc_f32_to_bf16(x)


def f32_to_f16_bits(x: float) -> int:
    return lib().orc_f32_to_f16(x)


# ---- fills -------------------------------------------------------------------
def fill_s4(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.int8)
    lib().orc_fill_s4(_ptr(out), n, seed)
    return out


def fill_s8(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.int8)
    lib().orc_fill_s8(_ptr(out), n, seed)
    return out


def fill_nibbles(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.uint8)
    lib().orc_fill_nibbles(_ptr(out), n, seed)
    return out


def fill_e2m1_bitcast(n: int, seed: int):
    q = np.empty(n, np.int8)
    bc = np.empty(n, np.int8)
    lib().orc_fill_e2m1_bitcast(_ptr(q), _ptr(bc), n, seed)
    return q, bc


def fill_rmsnorm_x(n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_fill_rmsnorm_x(_ptr(out), n)
    return out


# ---- layouts -----------------------------------------------------------------
def unpack_i32_nibbles_first(a: np.ndarray) -> np.ndarray:
    a = _c(a, np.int32)
    out = np.empty((a.shape[0] * 8, a.shape[1]), np.int16)
    lib().orc_unpack_i32_nibbles_first(_ptr(a), a.shape[0], a.shape[1], _ptr(out))
    return out


def unpack_i32_nibbles_last(a: np.ndarray) -> np.ndarray:
    a = _c(a, np.int32)
    out = np.empty((a.shape[0], a.shape[1] * 8), np.int16)
    lib().orc_unpack_i32_nibbles_last(_ptr(a), a.shape[0], a.shape[1], _ptr(out))
    return out


def pack_i32_nibbles_first(u: np.ndarray) -> np.ndarray:
    u = _c(u, np.uint8)
    K, N = u.shape
    out = np.empty((K // 8, N), np.int32)
    lib().orc_pack_i32_nibbles_first(_ptr(u), K, N, _ptr(out))
    return out


def pack_i32_nibbles_last(u: np.ndarray) -> np.ndarray:
    u = _c(u, np.uint8)
    R, C = u.shape
    out = np.empty((R, C // 8), np.int32)
    lib().orc_pack_i32_nibbles_last(_ptr(u), R, C, _ptr(out))
    return out


def pack_s4_along_k(b: np.ndarray) -> np.ndarray:
    b = _c(b, np.int8)
    K, N = b.shape
    out = np.empty((K // 2, N), np.uint8)
    lib().orc_pack_s4_along_k(_ptr(b), K, N, _ptr(out))
    return out


def pack_s4_rows(a: np.ndarray) -> np.ndarray:
    a = _c(a, np.int8)
    M, K = a.shape
    out = np.empty((M, K // 2), np.uint8)
    lib().orc_pack_s4_rows(_ptr(a), M, K, _ptr(out))
    return out


# ---- GEMMs -------------------------------------------------------------------
def s32_gemm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = _c(a, np.int8)
    b = _c(b, np.int8)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.int32)
    lib().orc_s32_gemm(_ptr(a), _ptr(b), _ptr(c), m, n, k)
    return c


def gptq_s4a_gemm(a_s4, a_scale, b_s4, s_f16_bits, gs: int) -> np.ndarray:
    """Reference formula (dpas_s4_gptq_sc.cpp:273-288); returns fp16 bits [m, n]."""
    a = _c(a_s4, np.int8)
    b = _c(b_s4, np.int8)
    asc = _c(a_scale, np.float32)
    s = _c(s_f16_bits, np.uint16)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.uint16)
    lib().orc_gptq_s4a_gemm(_ptr(a), _ptr(asc), _ptr(b), _ptr(s), m, n, k, gs, _ptr(c))
    return c


def nvfp4_lut_gemm_s8a(a_s8, packed, a_s, b_s) -> np.ndarray:
    """Reference formula (nibble_lut_sc.cpp:319-330); returns fp16 bits [m, n]."""
    a = _c(a_s8, np.int8)
    p = _c(packed, np.uint8)
    m, k = a.shape
    n = p.shape[1]
    c = np.empty((m, n), np.uint16)
    lib().orc_nvfp4_lut_gemm_s8a(_ptr(a), _ptr(p), _ptr(_c(a_s, np.float32)), _ptr(_c(b_s, np.float32)),
                                 m, n, k, _ptr(c))
    return c


def gptq_dequant(qweight, qzeros, scales_f16_bits, g_idx, K, N, group_size, zero_offset=1):
    qw = _c(qweight, np.int32)
    qz = None if qzeros is None else _c(qzeros, np.int32)
    sc = _c(scales_f16_bits, np.uint16)
    gi = None if g_idx is None else _c(g_idx, np.int32)
    w = np.empty((K, N), np.float32)
    lib().orc_gptq_dequant(_ptr(qw), _ptr(qz), _ptr(sc), _ptr(gi), K, N, group_size, zero_offset, _ptr(w))
    return w


def gptq_gemm(a, qweight, qzeros, scales_f16_bits, g_idx, M, N, K, group_size, zero_offset=1, threads=0):
    a = _c(a, np.float32)
    qw = _c(qweight, np.int32)
    qz = None if qzeros is None else _c(qzeros, np.int32)
    sc = _c(scales_f16_bits, np.uint16)
    gi = None if g_idx is None else _c(g_idx, np.int32)
    c = np.empty((M, N), np.float32)
    lib().orc_gptq_gemm(_ptr(a), _ptr(qw), _ptr(qz), _ptr(sc), _ptr(gi), M, N, K, group_size, zero_offset,
                        _ptr(c), threads)
    return c


def gptq_act_order_perm(g_idx, group_size: int) -> np.ndarray:
    gi = _c(g_idx, np.int32)
    perm = np.empty_like(gi)
    lib().orc_gptq_act_order_perm(_ptr(gi), gi.shape[0], group_size, _ptr(perm))
    return perm


def nvfp4_dequant(w, layout, scale, scale_kind, global_scale, K, N):
    w = _c(w, np.uint8)
    scale = np.ascontiguousarray(scale)
    out = np.empty((K, N), np.float32)
    lib().orc_nvfp4_dequant(_ptr(w), layout, _ptr(scale), scale_kind, float(global_scale), K, N, _ptr(out))
    return out


def nvfp4_gemm(a, w, layout, scale, scale_kind, global_scale, M, N, K, threads=0):
    a = _c(a, np.float32)
    w = _c(w, np.uint8)
    scale = np.ascontiguousarray(scale)
    c = np.empty((M, N), np.float32)
    lib().orc_nvfp4_gemm(_ptr(a), _ptr(w), layout, _ptr(scale), scale_kind, float(global_scale), M, N, K,
                         _ptr(c), threads)
    return c


def nvfp4_quant_act(a, global_dec: float):
    a = _c(a, np.float32)
    M, K = a.shape
    codes = np.empty((M, K // 2), np.uint8)
    sf = np.empty((M, K // 16), np.uint8)
    lib().orc_nvfp4_quant_act(_ptr(a), M, K, float(global_dec), _ptr(codes), _ptr(sf))
    return codes, sf


def nvfp4_act_dequant(codes, sf, global_dec: float, M: int, K: int):
    out = np.empty((M, K), np.float32)
    lib().orc_nvfp4_act_dequant(_ptr(_c(codes, np.uint8)), _ptr(_c(sf, np.uint8)), float(global_dec), M, K,
                                _ptr(out))
    return out


def rmsnorm_quant_s8(x, eps: float = 1e-6):
    x = _c(x, np.float32)
    m, k = x.shape
    q = np.empty((m, k), np.int8)
    s = np.empty(m, np.float32)
    lib().orc_rmsnorm_quant_s8(_ptr(x), _ptr(q), _ptr(s), m, k, eps)
    return q, s


def rmsnorm_nvfp4(x, gamma, eps: float, global_dec: float):
    """-> (codes u8 [M, K/2], sf u8 [M, K/16]) of the fused RMSNorm -> NVFP4 producer."""
    x = _c(x, np.float32)
    m, k = x.shape
    g = None if gamma is None else _c(gamma, np.float32)
    codes = np.empty((m, k // 2), np.uint8)
    sf = np.empty((m, k // 16), np.uint8)
    lib().orc_rmsnorm_nvfp4(_ptr(x), None if g is None else _ptr(g), m, k, float(eps), float(global_dec),
                            _ptr(codes), _ptr(sf))
    return codes, sf


def rowscale_fp8(y):
    y = _c(y, np.float32)
    M, N = y.shape
    q = np.empty((M, N), np.uint8)
    s = np.empty(M, np.float32)
    lib().orc_rowscale_fp8(_ptr(y), M, N, _ptr(q), _ptr(s))
    return q, s


# ---- metrics -----------------------------------------------------------------
def cosine(x, y) -> float:
    x = _c(x, np.float32).ravel()
    y = _c(y, np.float32).ravel()
    return lib().orc_cosine(_ptr(x), _ptr(y), x.size)


def max_abs(x, y) -> float:
    x = _c(x, np.float32).ravel()
    y = _c(y, np.float32).ravel()
    return lib().orc_max_abs(_ptr(x), _ptr(y), x.size)


def rel_frob(got, ref) -> float:
    g = _c(got, np.float32).ravel()
    r = _c(ref, np.float32).ravel()
    return lib().orc_rel_frob(_ptr(g), _ptr(r), g.size)
