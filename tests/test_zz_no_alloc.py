"""w4_gptq_gemm_fp8_noalloc: the fp8 row-scaled GPTQ GEMM for callers that cannot
allocate device memory (its scratch is a static device array in libw4, not a
caller workspace).  Checked through the C ABI against w4_gptq_gemm with a
workspace and against the CPU oracle, on calls in a row at decode and prefill
token counts.  Kept in its own file, collected last."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from tests._util import assert_gemm_close, bits16, f32, np_
from xe2x2_b200 import _lib as L
from xe2x2_b200 import synth

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _existing(lib, a, qw, qz, sc, M, N, K, st):
    q = torch.empty((M, N), dtype=torch.uint8, device=a.device)
    rs = torch.empty(M, dtype=torch.float32, device=a.device)
    nb = lib.w4_gptq_workspace_bytes(M, N, K, 128, 0, L.W4_E4M3)
    ws = torch.zeros(nb, dtype=torch.uint8, device=a.device)  # the sync area starts zeroed
    rc = lib.w4_gptq_gemm(_p(a), L.W4_BF16, _p(qw), _p(qz), _p(sc), None, _p(q), L.W4_E4M3, _p(rs),
                          M, N, K, 128, 1, _p(ws), nb, st)
    assert rc == L.W4_OK, lib.w4_last_error()
    return q, rs


def _noalloc(lib, a, qw, qz, sc, M, N, K, st):
    q = torch.empty((M, N), dtype=torch.uint8, device=a.device)
    rs = torch.empty(M, dtype=torch.float32, device=a.device)
    rc = lib.w4_gptq_gemm_fp8_noalloc(_p(a), L.W4_BF16, _p(qw), _p(qz), _p(sc), _p(q), _p(rs),
                                      M, N, K, 128, 1, st)
    assert rc == L.W4_OK, lib.w4_last_error()
    return q, rs


def _dequant(q, rs):
    return f32(q.view(torch.float8_e4m3fn)) * np_(rs)[:, None]


def test_noalloc_matches_workspace_entry_point(cuda):
    """The entry point without a workspace runs its GEMM without a K split, the one with a
    workspace may split K over CTAs: the same fp32 product up to the order of its sums, so
    row scales agree to fp32 rounding and the e4m3 codes to one code step."""
    lib = L.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    K, N = 2048, 1024
    qw, qz, sc, _ = synth.gptq_weights(K, N, 128, asym=True, seed=21, device=cuda)
    ref_w = O.gptq_dequant(np_(qw), np_(qz), bits16(sc), None, K, N, 128, 1)
    # calls in a row: decode sizes (the decode GEMM) and M = 64 (the tensor-core GEMM)
    for call, M in enumerate((16, 5, 64, 1)):
        a = synth.activations(M, K, torch.bfloat16, seed=30 + call, device=cuda)
        q_ref, rs_ref = _existing(lib, a, qw, qz, sc, M, N, K, st)
        q, rs = _noalloc(lib, a, qw, qz, sc, M, N, K, st)
        torch.cuda.synchronize()
        assert np.isfinite(np_(rs)).all()
        np.testing.assert_allclose(np_(rs), np_(rs_ref), rtol=1e-5, atol=0)
        d, d_ref = _dequant(q, rs), _dequant(q_ref, rs_ref)
        # one e4m3 step is at most 1/8 of the value (2^-9 of the row maximum near zero)
        tol = np.abs(d_ref) / 8 + np_(rs_ref)[:, None] * 2.0 ** -9 + 1e-30
        assert (np.abs(d - d_ref) <= tol).all()
        # and both track the fp32 oracle within fp8 precision
        oracle = f32(a) @ ref_w
        assert_gemm_close(d, oracle, rel=5e-2, nmax=7e-2)


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    lib = L.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    K, N, M = 256, 1 << 16, 32  # M*N = 2 Mi elements > 1 Mi
    x = torch.empty(16, dtype=torch.uint8, device=cuda)
    rc = lib.w4_gptq_gemm_fp8_noalloc(_p(x), L.W4_BF16, _p(x), None, _p(x), _p(x), _p(x), M, N, K, 128, 1, st)
    assert rc == L.W4_ERR_UNSUPPORTED
    assert b"static scratch" in lib.w4_last_error()
