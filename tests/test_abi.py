"""C-ABI surface checks that need no GPU: the library loads, exports every
entry point declared in include/w4.h, and rejects bad arguments synchronously
(before any CUDA call)."""
import ctypes

import pytest

from xe2x2_b200 import _lib as L


def test_library_exports_every_header_symbol():
    lib = L.lib()
    names = L.header_symbols()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"missing exports: {missing}"
    # and every header symbol has a ctypes signature in the binding
    assert set(names) <= set(L._SIGS), set(names) - set(L._SIGS)


def test_version_and_status_strings():
    lib = L.lib()
    assert lib.w4_abi_version() == 1
    assert lib.w4_status_string(L.W4_OK) == b"ok"
    assert lib.w4_status_string(L.W4_ERR_UNSUPPORTED) == b"unsupported shape or option"


def _fake(addr=0x10000):
    return ctypes.c_void_p(addr)


def test_gptq_gemm_rejects_bad_arguments_without_gpu():
    lib = L.lib()
    # null qweight
    rc = lib.w4_gptq_gemm(_fake(), L.W4_F16, None, None, _fake(), None, _fake(), L.W4_F16, None,
                          1, 64, 128, 128, 1, None, 0, None)
    assert rc == L.W4_ERR_INVALID and b"qweight" in lib.w4_last_error()
    # K not a multiple of group size
    rc = lib.w4_gptq_gemm(_fake(), L.W4_F16, _fake(), None, _fake(), None, _fake(), L.W4_F16, None,
                          1, 64, 200, 128, 1, None, 0, None)
    assert rc == L.W4_ERR_INVALID
    # M < 1 (the reference harness rejects m < 1, dpas_s4_gptq_sc.cpp:239)
    rc = lib.w4_gptq_gemm(_fake(), L.W4_F16, _fake(), None, _fake(), None, _fake(), L.W4_F16, None,
                          0, 64, 128, 128, 1, None, 0, None)
    assert rc == L.W4_ERR_INVALID
    # ragged N (the reference requires n % tile == 0)
    rc = lib.w4_gptq_gemm(_fake(), L.W4_F16, _fake(), None, _fake(), None, _fake(), L.W4_F16, None,
                          1, 40, 128, 128, 1, None, 0, None)
    assert rc == L.W4_ERR_UNSUPPORTED
    # fp8 output without a row-scale buffer
    rc = lib.w4_gptq_gemm(_fake(), L.W4_F16, _fake(), None, _fake(), None, _fake(), L.W4_E4M3, None,
                          1, 64, 128, 128, 1, None, 0, None)
    assert rc == L.W4_ERR_INVALID
    # misaligned activation pointer
    rc = lib.w4_gptq_gemm(_fake(0x10002), L.W4_F16, _fake(), None, _fake(), None, _fake(), L.W4_F16,
                          None, 1, 64, 128, 128, 1, None, 0, None)
    assert rc == L.W4_ERR_INVALID
    # workspace too small for act_order
    rc = lib.w4_gptq_gemm(_fake(), L.W4_F16, _fake(), None, _fake(), _fake(), _fake(), L.W4_F16, None,
                          1, 64, 128, 128, 1, None, 0, None)
    assert rc == L.W4_ERR_INVALID and b"workspace" in lib.w4_last_error()


def test_workspace_sizes():
    lib = L.lib()
    sync = L.W4_WORKSPACE_SYNC_BYTES
    assert f"#define W4_WORKSPACE_SYNC_BYTES {sync}" in open(L.HEADER).read()
    # every workspace starts with the zeroed sync area
    assert lib.w4_gptq_workspace_bytes(16, 4096, 4096, 128, 0, L.W4_F16) >= sync
    assert lib.w4_gptq_workspace_bytes(16, 4096, 4096, 128, 1, L.W4_F16) >= sync + 16 * 4096 * 2
    assert lib.w4_gptq_workspace_bytes(16, 4096, 4096, 128, 0, L.W4_E4M3) >= sync + 16 * 4096 * 4
    # the NVFP4 decode GEMM's K-split partials (20 column tiles of 256 are too few for the SMs)
    dec4 = lib.w4_nvfp4_workspace_bytes(8, 5120, 5120, L.W4_ACT_W4A16, L.W4_BF16) - sync
    assert dec4 >= 2 * 8 * 5120 * 4 and dec4 % 256 == 0
    assert lib.w4_nvfp4_gemm_q_workspace_bytes(128, 256, 256, L.W4_E4M3_ATOMS, L.W4_BF16) >= sync
    # the decode GEMM's K-split partials (4-column tiles too few for the SMs): config 1 shape
    dec = lib.w4_gptq_workspace_bytes(16, 4096, 4096, 128, 0, L.W4_F16) - sync
    assert dec >= 2 * 16 * 4096 * 4 and dec % 256 == 0
    # from 9 tokens the W4A16 tensor-core GEMM splits K over CTAs for few output tiles
    assert lib.w4_nvfp4_workspace_bytes(16, 5120, 5120, L.W4_ACT_W4A16, L.W4_BF16) % 256 == 0


def test_nvfp4_rejects_bad_arguments_without_gpu():
    lib = L.lib()
    # e4m3 scales need a tensor scale
    rc = lib.w4_nvfp4_gemm(_fake(), _fake(), L.W4_NVFP4_NK, _fake(), L.W4_E4M3, None, L.W4_ACT_W4A16, None,
                           _fake(), L.W4_BF16, None, 1, 64, 128, None, 0, None)
    assert rc == L.W4_ERR_INVALID
    # the GEMM reads the NK layout only
    rc = lib.w4_nvfp4_gemm(_fake(), _fake(), L.W4_NVFP4_KN, _fake(), L.W4_E4M3, _fake(), L.W4_ACT_W4A16,
                           None, _fake(), L.W4_BF16, None, 1, 64, 128, None, 0, None)
    assert rc == L.W4_ERR_UNSUPPORTED and b"repack" in lib.w4_last_error()
    rc = lib.w4_rmsnorm_quant_s8(_fake(), _fake(), _fake(), 1, 12, 1e-6, None)
    assert rc == L.W4_ERR_INVALID


def test_oracle_library_loads():
    import oracle as O
    assert O.e2m1_value(7) == 6.0


def test_launch_overlap_mode_round_trip():
    lib = L.lib()
    old = lib.w4_get_launch_overlap()
    assert old == L.W4_OVERLAP_DEPENDENT  # the default
    try:
        for m in (L.W4_OVERLAP_OFF, L.W4_OVERLAP_STATIC_WEIGHTS, L.W4_OVERLAP_DEPENDENT):
            assert lib.w4_set_launch_overlap(m) == L.W4_OK
            assert lib.w4_get_launch_overlap() == m
        assert lib.w4_set_launch_overlap(3) == L.W4_ERR_INVALID
        assert lib.w4_get_launch_overlap() == L.W4_OVERLAP_DEPENDENT
    finally:
        lib.w4_set_launch_overlap(old)


def test_producer_and_prequantised_gemm_reject_bad_arguments_without_gpu():
    lib = L.lib()
    f = _fake()
    # K not a multiple of 64
    assert lib.w4_rmsnorm_quant_nvfp4(f, L.W4_BF16, None, 1e-6, f, f, f, 4, 96, None) == L.W4_ERR_INVALID
    # fp32 input
    assert lib.w4_rmsnorm_quant_nvfp4(f, L.W4_F32, None, 1e-6, f, f, f, 4, 128, None) == L.W4_ERR_INVALID
    # negative eps
    assert lib.w4_rmsnorm_quant_nvfp4(f, L.W4_BF16, None, -1.0, f, f, f, 4, 128, None) == L.W4_ERR_INVALID
    assert lib.w4_nvfp4_act_codes_bytes(200, 1024) == 256 * 512  # rows padded to the 128-row tile
    # the pre-quantised GEMM: bf16 (folded) weight scales cannot feed the block-scaled MMA
    rc = lib.w4_nvfp4_gemm_q(f, f, f, f, L.W4_NVFP4_NK, f, L.W4_BF16, None, f, L.W4_BF16, None, 128, 256,
                             1024, None, 0, None)
    assert rc == L.W4_ERR_UNSUPPORTED
    # K not a multiple of 256
    rc = lib.w4_nvfp4_gemm_q(f, f, f, f, L.W4_NVFP4_NK, f, L.W4_E4M3, f, f, L.W4_BF16, None, 128, 256,
                             640, None, 0, None)
    assert rc == L.W4_ERR_UNSUPPORTED
    # missing activation scale atoms
    rc = lib.w4_nvfp4_gemm_q(f, None, f, f, L.W4_NVFP4_NK, f, L.W4_E4M3, f, f, L.W4_BF16, None, 128, 256,
                             1024, None, 0, None)
    assert rc == L.W4_ERR_INVALID


def test_tp_option_needs_a_communicator():
    assert L.lib().w4_tp_set_fused_epilogue(None, 1) == L.W4_ERR_INVALID


def test_python_wrappers_refuse_cpu_tensors_and_missing_scales():
    import torch

    from xe2x2_b200 import ops

    x = torch.zeros(2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.rmsnorm_quant_nvfp4(x, torch.ones(1))
    w = torch.zeros(64, 32, dtype=torch.uint8)
    with pytest.raises(ValueError):
        ops.NVFP4Linear(w, torch.zeros(8, 32, dtype=torch.uint8), torch.ones(1), None, L.W4_ACT_NVFP4)


def test_grouped_gemm_checks_offsets_without_gpu():
    import ctypes
    lib = L.lib()
    f = _fake()
    for off in ((1, 2, 4), (0, 3, 2)):
        arr = (ctypes.c_int32 * 3)(*off)
        assert lib.w4_gptq_gemm_grouped_workspace_bytes(arr, 2, 64, 256, 128, L.W4_BF16) == 0
        rc = lib.w4_gptq_gemm_grouped(f, L.W4_BF16, f, None, f, arr, 2, f, L.W4_BF16, None, 64, 256, 128, 1, f,
                                      1 << 20, None)
        assert rc == L.W4_ERR_INVALID and b"offsets" in lib.w4_last_error()
        rc = lib.w4_nvfp4_gemm_grouped(f, f, f, f, arr, 2, f, L.W4_BF16, None, 64, 256, f, 1 << 20, None)
        assert rc == L.W4_ERR_INVALID
    ok = (ctypes.c_int32 * 9)(0, 3, 3, 4, 11, 13, 29, 34, 35)
    assert lib.w4_gptq_gemm_grouped_workspace_bytes(ok, 8, 1856, 2688, 128, L.W4_BF16) >= L.W4_WORKSPACE_SYNC_BYTES
    assert lib.w4_nvfp4_gemm_grouped_workspace_bytes(ok, 8, 2688, 1856, L.W4_E4M3) >= \
        L.W4_WORKSPACE_SYNC_BYTES + 35 * 2688 * 4


def test_read_probe_rejects_bad_arguments_without_gpu():
    lib = L.lib()
    f = _fake()
    assert lib.w4_read_probe(None, 1024, f, None) == L.W4_ERR_INVALID
    assert lib.w4_read_probe(f, 1000, f, None) == L.W4_ERR_INVALID  # not a multiple of 16
    assert lib.w4_read_probe(_fake(0x10008), 1024, f, None) == L.W4_ERR_INVALID  # misaligned
    assert b"aligned" in lib.w4_last_error()
