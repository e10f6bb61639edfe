"""ctypes binding of libw4.so (the C ABI declared in include/w4.h).

There is no CPU fallback: if the library cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import re

from . import build as _build

_lib = None

# status codes / enums (include/w4.h)
W4_OK, W4_ERR_INVALID, W4_ERR_UNSUPPORTED, W4_ERR_CUDA, W4_ERR_TIMEOUT, W4_ERR_NCCL = range(6)
W4_F16, W4_BF16, W4_F32, W4_E4M3, W4_S8, W4_E4M3_ATOMS = range(6)
W4_NVFP4_KN, W4_NVFP4_NK = 0, 1
W4_ACT_W4A16, W4_ACT_NVFP4 = 0, 1
W4_TP_COLUMN, W4_TP_ROW = 0, 1
W4_OVERLAP_OFF, W4_OVERLAP_DEPENDENT, W4_OVERLAP_STATIC_WEIGHTS = 0, 1, 2
W4_TP_UNIQUE_ID_BYTES = 128
W4_WORKSPACE_SYNC_BYTES = 16384  # zeroed sync area at the start of every workspace

HEADER = os.path.join(os.path.dirname(_build.HERE), "include", "w4.h")


class W4Error(RuntimeError):
    def __init__(self, status: int, fn: str, detail: str):
        self.status = status
        super().__init__(f"{fn} failed: status {status}: {detail}")


_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t

_SIGS = {
    "w4_abi_version": (_I, []),
    "w4_status_string": (ctypes.c_char_p, [_I]),
    "w4_last_error": (ctypes.c_char_p, []),
    "w4_check_device_status": (_I, []),
    "w4_set_launch_overlap": (_I, [_I]),
    "w4_get_launch_overlap": (_I, []),
    "w4_decode_fallback_count": (ctypes.c_ulonglong, []),
    "w4_read_probe": (_I, [_P, _Z, _P, _P]),
    "w4_gptq_dequant": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "w4_gptq_repack_act_order": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
    "w4_gptq_workspace_bytes": (_Z, [_I, _I, _I, _I, _I, _I]),
    "w4_gptq_gemm": (_I, [_P, _I, _P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P, _Z, _P]),
    "w4_gptq_gemm_grouped_workspace_bytes": (_Z, [_P, _I, _I, _I, _I, _I]),
    "w4_gptq_gemm_grouped": (_I, [_P, _I, _P, _P, _P, _P, _I, _P, _I, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "w4_nvfp4_gemm_grouped_workspace_bytes": (_Z, [_P, _I, _I, _I, _I]),
    "w4_nvfp4_gemm_grouped": (_I, [_P, _P, _P, _P, _P, _I, _P, _I, _P, _I, _I, _P, _Z, _P]),
    "w4_gptq_gemm_s4a": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "w4_gptq_gemm_fp8_noalloc": (_I, [_P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "w4_nvfp4_dequant": (_I, [_P, _I, _P, _I, _P, _I, _I, _P, _P]),
    "w4_nvfp4_quant_act": (_I, [_P, _I, _I, _P, _P, _P, _P]),
    "w4_nvfp4_workspace_bytes": (_Z, [_I, _I, _I, _I, _I]),
    "w4_nvfp4_gemm": (_I, [_P, _P, _I, _P, _I, _P, _I, _P, _P, _I, _P, _I, _I, _I, _P, _Z, _P]),
    "w4_nvfp4_repack_kn_to_nk": (_I, [_P, _I, _I, _P, _P]),
    "w4_nvfp4_scale_atoms_bytes": (_Z, [_I, _I]),
    "w4_nvfp4_repack_scales": (_I, [_P, _I, _I, _P, _P]),
    "w4_nvfp4_act_codes_bytes": (_Z, [_I, _I]),
    "w4_rmsnorm_quant_nvfp4": (_I, [_P, _I, _P, _F, _P, _P, _P, _I, _I, _P]),
    "w4_nvfp4_gemm_q_workspace_bytes": (_Z, [_I, _I, _I, _I, _I]),
    "w4_nvfp4_gemm_q": (_I, [_P, _P, _P, _P, _I, _P, _I, _P, _P, _I, _P, _I, _I, _I, _P, _Z, _P]),
    "w4_nvfp4_lut_gemm_s8a": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "w4_rmsnorm_quant_s8": (_I, [_P, _P, _P, _I, _I, _F, _P]),
    "w4_rowscale_fp8": (_I, [_P, _I, _P, _P, _I, _I, _P]),
    "w4_tp_get_unique_id": (_I, [_P]),
    "w4_tp_comm_init": (_I, [ctypes.POINTER(_P), _I, _I, _P, _I]),
    "w4_tp_comm_destroy": (_I, [_P]),
    "w4_tp_comm_abort": (_I, [_P]),
    "w4_tp_allreduce": (_I, [_P, _P, _Z, _I, _P]),
    "w4_tp_wait": (_I, [_P, _P, _I]),
    "w4_tp_set_fused_epilogue": (_I, [_P, _I]),
    "w4_tp_linear_workspace_bytes": (_Z, [_I, _I, _I, _I, _I, _I, _I]),
    "w4_tp_linear": (_I, [_P, _I, _P, _I, _P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P, _Z, _P]),
}


def header_symbols() -> list[str]:
    """Every function name declared in include/w4.h."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(w4_[a-z0-9_]+)\s*\(", text)))


def lib():
    """Load libw4.so (building it first if the sources are newer)."""
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call a status-returning entry point; raise W4Error on failure."""
    L = lib()
    rc = getattr(L, name)(*args)
    if rc != W4_OK:
        detail = (L.w4_last_error() or b"").decode() or L.w4_status_string(rc).decode()
        raise W4Error(rc, name, detail)


def loaded_path() -> str:
    return lib()._name
