"""Pins the CPU oracle to the reference's own known answers (CPU only).

* E2M1 bitcast-onto-s4 negative: the reference records max_abs 352 on its
  8x16x64 check tile and 1408 on the 256^3 tile (FINDINGS.md:936-951 of the
  reference; fills of kernels/nvfp4/bitcast_e2m1_s4.cpp:67-78).  Reproducing
  both numbers pins the fill formulas, the E2M1 code table and the integer GEMM.
* GPTQ unpack: fixtures produced by the reference's own unpackers
  (kernels/nvfp4/gptq_s4_dump.py:61-73) -- tests/golden/make_golden.py.
* NVFP4 LUT closure: LUT -> s8 is exact (max_abs 0, FINDINGS.md:280-294); GPTQ
  group-scale closure (cosine 1.0, FINDINGS.md:1066-1084).
* RMSNorm-s8 contract: codes within 1 of the float host oracle for f16 inputs
  (results/k5/SUMMARY.md:1-21).
"""
import os

import numpy as np
import pytest
import torch

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden", "gptq_unpack.npz")


@pytest.mark.parametrize("m,n,k,expect", [(8, 16, 64, 352), (256, 256, 256, 1408)])
def test_e2m1_bitcast_negative_matches_reference(m, n, k, expect):
    a = O.fill_s4(m * k, 1).reshape(m, k)
    q, bc = O.fill_e2m1_bitcast(k * n, 9)
    ref = O.s32_gemm(a, q.reshape(k, n)).astype(np.int64)
    got = O.s32_gemm(a, bc.reshape(k, n)).astype(np.int64)
    assert int(np.abs(ref - got).max()) == expect


def test_e2m1_table_is_twice_the_format_values():
    for nib in range(16):
        assert O.lib().orc_e2m1_q(nib) == int(2 * O.e2m1_value(nib))
    assert [O.e2m1_value(i) for i in range(8)] == [0, 0.5, 1, 1.5, 2, 3, 4, 6]


def test_gptq_unpack_matches_reference_unpackers():
    d = np.load(GOLD)
    for p in ("a", "b"):
        assert np.array_equal(O.unpack_i32_nibbles_first(d[f"{p}_qweight"]), d[f"{p}_unpack_first"])
        assert np.array_equal(O.unpack_i32_nibbles_last(d[f"{p}_qzeros"]), d[f"{p}_unpack_last"])
        # pack is the exact inverse
        u = d[f"{p}_unpack_first"].astype(np.uint8)
        assert np.array_equal(O.pack_i32_nibbles_first(u), d[f"{p}_qweight"])
        z = d[f"{p}_unpack_last"].astype(np.uint8)
        assert np.array_equal(O.pack_i32_nibbles_last(z), d[f"{p}_qzeros"])


def test_gptq_dequant_follows_reference_layout():
    """w = s * (u - (z + 1)) with u, z from the reference unpackers (v1 '+1' zeros)."""
    d = np.load(GOLD)
    qw = d["b_qweight"]  # [64, 24] -> K=512, N=24
    K, N, gs = qw.shape[0] * 8, qw.shape[1], 128
    rng = np.random.default_rng(3)
    qz_u = rng.integers(0, 16, size=(K // gs, N)).astype(np.uint8)
    qz = O.pack_i32_nibbles_last(qz_u)
    sc = (np.abs(rng.standard_normal((K // gs, N))) * 0.02 + 1e-3).astype(np.float16)
    u = d["b_unpack_first"].astype(np.float32)
    z = O.unpack_i32_nibbles_last(qz).astype(np.float32)
    g = np.arange(K) // gs
    expect = sc.astype(np.float32)[g] * (u - (z[g] + 1))
    got = O.gptq_dequant(qw, qz, sc.view(np.uint16), None, K, N, gs, 1)
    assert np.array_equal(got, expect)
    # symmetric: stored zero 7 + 1 == 8, i.e. the reference's s4 = u - 8 (gptq_s4_dump.py:114)
    got_sym = O.gptq_dequant(qw, None, sc.view(np.uint16), None, K, N, gs, 1)
    assert np.array_equal(got_sym, sc.astype(np.float32)[g] * d["b_s4"].astype(np.float32))


def test_gptq_s4a_formula_closure():
    """Reference check tile 8x16x128 and 8x256x256: exact integer group partials."""
    for (m, n, k) in [(8, 16, 128), (8, 256, 256)]:
        a = O.fill_s4(m * k, 1).reshape(m, k)
        b = O.fill_s4(k * n, 3).reshape(k, n)
        s = (np.linspace(0.0028, 0.0102, (k // 128) * n)).astype(np.float16).reshape(k // 128, n)
        asc = np.full(m, 0.02, np.float32)
        c = O.f16_bits_to_f32(O.gptq_s4a_gemm(a, asc, b, s.view(np.uint16), 128))
        ref = np.zeros((m, n), np.float64)
        for g in range(k // 128):
            part = a[:, g * 128:(g + 1) * 128].astype(np.int64) @ b[g * 128:(g + 1) * 128].astype(np.int64)
            ref += part * 0.02 * s[g].astype(np.float64)
        assert O.cosine(c, ref.astype(np.float32)) > 0.99999
        assert O.max_abs(c, ref.astype(np.float32)) < 1e-2 * np.abs(ref).max() + 1e-6


def test_nvfp4_lut_closure_exact():
    """LUT -> s8 GEMM equals the integer GEMM on 2*e2m1 codes (max_abs 0)."""
    m, n, k = 4, 64, 256
    a = O.fill_s8(m * k, 1).reshape(m, k)
    nib = O.fill_nibbles(k * n, 9).reshape(k, n)
    packed = np.zeros((k // 2, n), np.uint8)
    packed[:] = (nib[0::2] & 15) | ((nib[1::2] & 15) << 4)
    q = np.vectorize(lambda v: O.lib().orc_e2m1_q(int(v)))(nib).astype(np.int8)
    ints = O.s32_gemm(a, q).astype(np.float32)
    c = O.f16_bits_to_f32(O.nvfp4_lut_gemm_s8a(a, packed, np.ones(m, np.float32), np.ones(n, np.float32)))
    assert np.array_equal(c, ints.astype(np.float16).astype(np.float32))


def test_rmsnorm_s8_contract():
    """f16 input vs float host oracle: codes within 1 (reference acceptance bound)."""
    for (m, k) in [(1, 5120), (4, 17408)]:
        x = O.fill_rmsnorm_x(m * k).reshape(m, k)
        q_ref, s_ref = O.rmsnorm_quant_s8(x)
        x16 = x.astype(np.float16).astype(np.float32)
        q16, s16 = O.rmsnorm_quant_s8(x16)
        assert np.abs(q_ref.astype(np.int32) - q16.astype(np.int32)).max() <= 1
        assert np.all(s_ref > 0) and np.all(s16 > 0)
    q0, s0 = O.rmsnorm_quant_s8(np.zeros((2, 64), np.float32))
    assert np.all(q0 == 0) and np.all(s0 == 1.0)


def test_codecs_match_torch():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(20000) * 200).astype(np.float32)
    inr = np.abs(x) < 448
    mine = np.array([O.e4m3_from_f32(float(v)) for v in x], np.uint8)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mine[inr], ref[inr])
    assert all(O.e4m3_from_f32(float(v)) & 0x7F == 0x7E for v in x[~inr])  # saturating
    for b in range(256):
        if b & 0x7F == 0x7F:
            continue
        assert O.e4m3_from_f32(O.e4m3_value(b)) == b or b == 0x80
    h = (rng.standard_normal(20000) * 1000).astype(np.float32)
    assert np.array_equal(np.array([O.f32_to_f16_bits(float(v)) for v in h], np.uint16),
                          h.astype(np.float16).view(np.uint16))
    assert np.array_equal(np.array([O.f32_to_bf16_bits(float(v)) for v in h], np.uint16),
                          torch.from_numpy(h).to(torch.bfloat16).view(torch.uint16).numpy())


def test_e2m1_rounding_is_nearest_even():
    cands = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6])
    for v in np.linspace(-7, 7, 2801):
        c = O.e2m1_from_f32(float(v))
        a = min(abs(v), 6.0)
        assert abs(abs(O.e2m1_value(c)) - a) <= np.min(np.abs(cands - a)) + 1e-7
    # ties go to the code with an even mantissa bit
    for v, want in [(0.25, 0.0), (0.75, 1.0), (1.25, 1.0), (1.75, 2.0), (2.5, 2.0), (3.5, 4.0), (5.0, 4.0)]:
        assert O.e2m1_value(O.e2m1_from_f32(v)) == want


def test_nvfp4_act_quant_roundtrip_error():
    rng = np.random.default_rng(1)
    a = rng.standard_normal((8, 256)).astype(np.float32)
    gdec = float(np.abs(a).max() / (448.0 * 6.0))
    codes, sf = O.nvfp4_quant_act(a, gdec)
    back = O.nvfp4_act_dequant(codes, sf, gdec, 8, 256)
    assert O.rel_frob(back, a) < 0.15  # 4-bit elements: ~10% error by design


def test_act_order_perm_is_stable_argsort():
    rng = np.random.default_rng(2)
    K, gs = 512, 128
    g_idx = np.empty(K, np.int32)
    g_idx[rng.permutation(K)] = np.arange(K) // gs
    perm = O.gptq_act_order_perm(g_idx, gs)
    assert np.array_equal(perm, np.argsort(g_idx, kind="stable"))


def test_gptq_gemm_oracle_group_partial_form():
    """The W4A16 oracle equals a float64 GEMM on dequantised weights to fp32 accuracy."""
    rng = np.random.default_rng(4)
    M, K, N, gs = 3, 256, 64, 128
    u = rng.integers(0, 16, size=(K, N)).astype(np.uint8)
    qw = O.pack_i32_nibbles_first(u)
    qz = O.pack_i32_nibbles_last(rng.integers(0, 16, size=(K // gs, N)).astype(np.uint8))
    sc = (np.abs(rng.standard_normal((K // gs, N))) * 0.02 + 1e-3).astype(np.float16)
    a = rng.standard_normal((M, K)).astype(np.float32)
    w = O.gptq_dequant(qw, qz, sc.view(np.uint16), None, K, N, gs, 1)
    ref = a.astype(np.float64) @ w.astype(np.float64)
    got = O.gptq_gemm(a, qw, qz, sc.view(np.uint16), None, M, N, K, gs, 1)
    assert O.rel_frob(got, ref.astype(np.float32)) < 1e-5
