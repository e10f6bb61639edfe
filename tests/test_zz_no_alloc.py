"""w4_gptq_gemm_fp8_noalloc: the fp8 row-scaled GPTQ GEMM for callers that cannot
allocate device memory (its scratch is a static device array in libw4, not a
caller workspace).  Checked through the C ABI against w4_gptq_gemm with a
workspace, on two calls in a row.  Kept in its own file, collected last."""
import ctypes

import numpy as np
import pytest
import torch

from xe2x2_b200 import _lib as L
from xe2x2_b200 import synth

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _existing(lib, a, qw, qz, sc, M, N, K, st):
    q = torch.empty((M, N), dtype=torch.uint8, device=a.device)
    rs = torch.empty(M, dtype=torch.float32, device=a.device)
    nb = lib.w4_gptq_workspace_bytes(M, N, K, 128, 0, L.W4_E4M3)
    ws = torch.empty(nb, dtype=torch.uint8, device=a.device)
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


def test_noalloc_matches_workspace_entry_point(cuda):
    lib = L.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    K, N = 2048, 1024
    qw, qz, sc, _ = synth.gptq_weights(K, N, 128, asym=True, seed=21, device=cuda)
    for call, M in enumerate((16, 5)):  # two calls in a row, different sizes
        a = synth.activations(M, K, torch.bfloat16, seed=30 + call, device=cuda)
        q_ref, rs_ref = _existing(lib, a, qw, qz, sc, M, N, K, st)
        q, rs = _noalloc(lib, a, qw, qz, sc, M, N, K, st)
        torch.cuda.synchronize()
        # same kernels and inputs: the cast is bit-exact, as in the workspace path's tests
        assert torch.equal(q, q_ref)
        assert torch.equal(rs, rs_ref)
        assert np.isfinite(rs.cpu().numpy()).all()


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    lib = L.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    K, N, M = 256, 1 << 16, 32  # M*N = 2 Mi elements > 1 Mi
    x = torch.empty(16, dtype=torch.uint8, device=cuda)
    rc = lib.w4_gptq_gemm_fp8_noalloc(_p(x), L.W4_BF16, _p(x), None, _p(x), _p(x), _p(x), M, N, K, 128, 1, st)
    assert rc == L.W4_ERR_UNSUPPORTED
    assert b"static scratch" in lib.w4_last_error()
