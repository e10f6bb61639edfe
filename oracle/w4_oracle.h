/*
 * w4_oracle.h -- CPU oracle for the weight-only quantized linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA
 * library (libw4) is compared against.  Only tests/, __graft_entry__.smoke()
 * and the cpu_baseline / --impl reference legs of bench.py may load it.  The
 * product path (xe2x2_b200/, include/w4.h) never links or calls it.
 *
 * It restates, in plain C, the host-side loops of the reference lab
 * hotschmoe/xe2x2 (paths below are relative to that project):
 *   - GPTQ checkpoint unpack      kernels/nvfp4/gptq_s4_dump.py:61-73,106-114
 *   - s4 pair packing             kernels/esimd_dpas/dpas_s4_gptq.cpp:46-66
 *   - deterministic fills         dpas_s4_gptq.cpp:50-53, nibble_lut_sc.cpp:59-67,
 *                                 epilogue_quant/rmsnorm_epilogue.cpp:176-177
 *   - GPTQ s4 host oracle         kernels/esimd_dpas/dpas_s4_gptq_sc.cpp:273-288
 *   - s32 host GEMM               kernels/nvfp4/bitcast_e2m1_s4.cpp:95-104
 *   - E2M1 table / nibble decode  kernels/nvfp4/nibble_lut_sc.cpp:42,70-92
 *   - NVFP4 LUT host oracle       kernels/nvfp4/nibble_lut_sc.cpp:319-330
 *   - RMSNorm + s8 host oracle    kernels/epilogue_quant/rmsnorm_epilogue.cpp:39-70
 *   - cosine / max_abs metrics    dpas_s4_gptq_sc.cpp:312-327
 * and, where the reference has no host code (E4M3 block scales, the W4A16
 * GEMM with real-valued activations, NVFP4 activation quantisation, the
 * fp8 row-scale cast), the published format definitions quoted in
 * results/literature/nvfp4-vs-ocp-mx.md:9-60.
 */
#ifndef W4_ORACLE_H
#define W4_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar format helpers (IEEE round-to-nearest-even) ---- */
float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);
float orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float f);
float orc_e2m1_value(uint8_t nib);
uint8_t orc_e2m1_from_f32(float x);      /* RNE, saturates to +-6 */
float orc_e4m3_value(uint8_t b);         /* 0x7F / 0xFF are NaN */
uint8_t orc_e4m3_from_f32(float x);      /* RNE, saturates to +-448 */
int8_t orc_e2m1_q(uint8_t nib);          /* 2*e2m1: nibble_lut_sc.cpp:70-75 */
int8_t orc_bitcast_nibble_s4(uint8_t nib); /* bitcast_e2m1_s4.cpp:60-65 */

/* ---- deterministic fills of the reference harnesses ---- */
void orc_fill_s4(int8_t *p, size_t n, unsigned seed);
void orc_fill_s8(int8_t *p, size_t n, unsigned seed);
void orc_fill_nibbles(uint8_t *p, size_t n, unsigned seed);
void orc_fill_e2m1_bitcast(int8_t *q, int8_t *bc, size_t n, unsigned seed);
void orc_fill_rmsnorm_x(float *p, size_t n);

/* ---- GPTQ layouts ---- */
void orc_unpack_i32_nibbles_first(const int32_t *a, int rows, int cols, int16_t *out);
void orc_unpack_i32_nibbles_last(const int32_t *a, int rows, int cols, int16_t *out);
void orc_pack_i32_nibbles_first(const uint8_t *u, int K, int N, int32_t *out);
void orc_pack_i32_nibbles_last(const uint8_t *u, int rows, int cols, int32_t *out);
void orc_pack_s4_along_k(const int8_t *b, int K, int N, uint8_t *out);
void orc_pack_s4_rows(const int8_t *a, int M, int K, uint8_t *out);

/* ---- integer / reference-formula GEMMs ---- */
void orc_s32_gemm(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k);
void orc_gptq_s4a_gemm(const int8_t *a, const float *a_scale, const int8_t *b,
                       const uint16_t *s_f16, int m, int n, int k, int gs,
                       uint16_t *c_f16);
void orc_nvfp4_lut_gemm_s8a(const int8_t *a, const uint8_t *packed, const float *a_s,
                            const float *b_s, int m, int n, int k, uint16_t *c_f16);

/* ---- W4A16 GPTQ ---- */
void orc_gptq_dequant(const int32_t *qweight, const int32_t *qzeros,
                      const uint16_t *scales_f16, const int32_t *g_idx, int K, int N,
                      int group_size, int zero_offset, float *w);
void orc_gptq_gemm(const float *a, const int32_t *qweight, const int32_t *qzeros,
                   const uint16_t *scales_f16, const int32_t *g_idx, int M, int N, int K,
                   int group_size, int zero_offset, float *c, int threads);
void orc_gptq_act_order_perm(const int32_t *g_idx, int K, int group_size, int32_t *perm);

/* ---- NVFP4 ---- */
#define ORC_NVFP4_KN 0 /* packed [K/2, N], two nibbles per byte along K (low = even k) */
#define ORC_NVFP4_NK 1 /* packed [N, K/2], K contiguous (low = even k) */
#define ORC_SCALE_E4M3 0
#define ORC_SCALE_BF16 1
void orc_nvfp4_dequant(const uint8_t *w, int layout, const uint8_t *scale, int scale_kind,
                       float global_scale, int K, int N, float *out);
void orc_nvfp4_gemm(const float *a, const uint8_t *w, int layout, const uint8_t *scale,
                    int scale_kind, float global_scale, int M, int N, int K, float *c,
                    int threads);
void orc_nvfp4_quant_act(const float *a, int M, int K, float global_dec, uint8_t *codes,
                         uint8_t *sf);
void orc_nvfp4_act_dequant(const uint8_t *codes, const uint8_t *sf, float global_dec,
                           int M, int K, float *out);

/* ---- epilogue quant ---- */
void orc_rmsnorm_quant_s8(const float *x, int8_t *q, float *scale, int m, int k, float eps);
void orc_rmsnorm_nvfp4(const float *x, const float *gamma, int m, int k, float eps, float global_dec,
                       uint8_t *codes, uint8_t *sf);
void orc_rowscale_fp8(const float *y, int M, int N, uint8_t *q, float *scale);

/* ---- metrics (dpas_s4_gptq_sc.cpp:312-327) ---- */
double orc_cosine(const float *x, const float *y, size_t n);
double orc_max_abs(const float *x, const float *y, size_t n);
double orc_rel_frob(const float *got, const float *ref, size_t n);

#ifdef __cplusplus
}
#endif
#endif
