/*
 * w4_oracle.c -- CPU oracle (test infrastructure only; see w4_oracle.h).
 *
 * Every function below restates a host loop of the reference lab
 * hotschmoe/xe2x2 (file:line given per function) or, where the reference has
 * no host code, the format definitions the reference quotes in
 * results/literature/nvfp4-vs-ocp-mx.md:9-60.  Arithmetic is fp32 with
 * round-to-nearest-even, in the same loop order as the reference where one
 * exists, so results are reproducible bit for bit on any IEEE host.
 */
#include "w4_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* threads > 0: use that many OpenMP threads; threads <= 0: all processors. */
static void set_threads(int threads) {
#ifdef _OPENMP
    omp_set_num_threads(threads > 0 ? threads : omp_get_num_procs());
#else
    (void)threads;
#endif
}

/* ------------------------------------------------------------------ */
/* scalar formats                                                      */
/* ------------------------------------------------------------------ */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    if (e == 0) {
        float v = (float)m * u2f(0x33800000u); /* m * 2^-24, exact */
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    return u2f(sign | ((e - 15 + 127) << 23) | (m << 13));
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    uint32_t a = x & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) return sign | 0x7C00 | (a > 0x7F800000u ? 0x200 : 0);
    if (a >= 0x477FF000u) return sign | 0x7C00; /* >= 65520 rounds to inf */
    if (a < 0x38800000u) {                      /* below 2^-14: subnormal */
        uint32_t e = a >> 23;
        if (e < 102) return sign;
        uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        int shift = 126 - (int)e;
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (a >> 23) - 127 + 15, m = a & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13), rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint16_t orc_f32_to_bf16(float f) {
    uint32_t x = f2u(f);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

/* E2M1: 1 sign, 2 exponent (bias 1), 1 mantissa; nvfp4-vs-ocp-mx.md:20-60 */
static const float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

float orc_e2m1_value(uint8_t nib) {
    float v = kE2M1[nib & 7];
    return (nib & 8) ? -v : v;
}

uint8_t orc_e2m1_from_f32(float x) {
    uint8_t s = (f2u(x) >> 31) ? 8 : 0;
    float a = fabsf(x);
    uint8_t c;
    /* midpoints tie to the code with an even (zero) mantissa bit */
    if (a <= 0.25f) c = 0;
    else if (a < 0.75f) c = 1;
    else if (a <= 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a <= 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a <= 5.0f) c = 6;
    else c = 7; /* saturate (also +-inf) */
    return (uint8_t)(s | c);
}

/* E4M3 ("fn"): bias 7, no infinity, NaN = S.1111.111, max 448. */
float orc_e4m3_value(uint8_t b) {
    uint32_t e = (b >> 3) & 0xF, m = b & 7;
    float v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0) v = (float)m * 0.001953125f; /* m * 2^-9 */
    else v = ldexpf(1.0f + (float)m / 8.0f, (int)e - 7);
    return (b & 0x80) ? -v : v;
}

uint8_t orc_e4m3_from_f32(float x) {
    uint32_t u = f2u(x);
    uint8_t s = (uint8_t)((u >> 24) & 0x80);
    uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return 0x7F;
    if (a >= 0x43E00000u) return (uint8_t)(s | 0x7E); /* >= 448: saturate */
    float af = u2f(a);
    if (a < 0x3C800000u) { /* below 2^-6: subnormal grid of 2^-9 */
        float q = nearbyintf(af * 512.0f); /* exact scaling, RNE */
        return (uint8_t)(s | (uint8_t)q);  /* q == 8 is the min normal code */
    }
    int e = (int)(a >> 23) - 127; /* -6 .. 8 */
    uint32_t m = a & 0x7FFFFFu;
    uint32_t q = m >> 20, rem = m & 0xFFFFFu;
    if (rem > 0x80000u || (rem == 0x80000u && (q & 1))) q++;
    uint32_t code = ((uint32_t)(e + 7) << 3) + q; /* carry into exponent is fine */
    if (code > 0x7E) code = 0x7E;
    return (uint8_t)(s | code);
}

/* kMag2 / nibble_to_q: kernels/nvfp4/nibble_lut_sc.cpp:42,70-75 */
int8_t orc_e2m1_q(uint8_t nib) {
    static const int8_t kMag2[8] = {0, 1, 2, 3, 4, 6, 8, 12};
    int8_t q = kMag2[nib & 7];
    return (nib & 8) ? (int8_t)-q : q;
}

/* bitcast_nibble_s4: kernels/nvfp4/bitcast_e2m1_s4.cpp:60-65 */
int8_t orc_bitcast_nibble_s4(uint8_t nib) {
    int v = nib & 15;
    return (int8_t)(v >= 8 ? v - 16 : v);
}

/* ------------------------------------------------------------------ */
/* deterministic fills                                                 */
/* ------------------------------------------------------------------ */
/* fill_s4: kernels/esimd_dpas/dpas_s4_gptq.cpp:50-53 */
void orc_fill_s4(int8_t *p, size_t n, unsigned seed) {
    for (size_t i = 0; i < n; ++i) p[i] = (int8_t)((int)((i * 17u + seed) % 16u) - 8);
}
/* fill_s8: kernels/nvfp4/nibble_lut_sc.cpp:59-62 */
void orc_fill_s8(int8_t *p, size_t n, unsigned seed) {
    for (size_t i = 0; i < n; ++i) p[i] = (int8_t)((int)((i * 17u + seed) % 129u) - 64);
}
/* fill_nibbles: kernels/nvfp4/nibble_lut_sc.cpp:64-67 */
void orc_fill_nibbles(uint8_t *p, size_t n, unsigned seed) {
    for (size_t i = 0; i < n; ++i) p[i] = (uint8_t)((i * 13u + seed) & 15u);
}
/* fill_e2m1_bitcast: kernels/nvfp4/bitcast_e2m1_s4.cpp:72-78 */
void orc_fill_e2m1_bitcast(int8_t *q, int8_t *bc, size_t n, unsigned seed) {
    for (size_t i = 0; i < n; ++i) {
        uint8_t nib = (uint8_t)((i * 13u + seed) & 15u);
        q[i] = orc_e2m1_q(nib);
        bc[i] = orc_bitcast_nibble_s4(nib);
    }
}
/* RMSNorm input: kernels/epilogue_quant/rmsnorm_epilogue.cpp:176-177 */
void orc_fill_rmsnorm_x(float *p, size_t n) {
    for (size_t i = 0; i < n; ++i) p[i] = (float)((int)((i * 17u) % 200u) - 100) * 0.02f;
}

/* ------------------------------------------------------------------ */
/* GPTQ layouts                                                        */
/* ------------------------------------------------------------------ */
/* unpack_i32_nibbles_first: kernels/nvfp4/gptq_s4_dump.py:69-73
 * a int32 [rows, cols] -> out [rows*8, cols]; nibble s of a[r][c] is row 8r+s. */
void orc_unpack_i32_nibbles_first(const int32_t *a, int rows, int cols, int16_t *out) {
    for (int r = 0; r < rows; ++r)
        for (int s = 0; s < 8; ++s)
            for (int c = 0; c < cols; ++c)
                out[((size_t)r * 8 + s) * cols + c] = (int16_t)(((uint32_t)a[(size_t)r * cols + c] >> (4 * s)) & 15u);
}
/* unpack_i32_nibbles_last: kernels/nvfp4/gptq_s4_dump.py:61-66
 * a int32 [rows, cols] -> out [rows, cols*8]; nibble s of a[r][c] is column 8c+s. */
void orc_unpack_i32_nibbles_last(const int32_t *a, int rows, int cols, int16_t *out) {
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c)
            for (int s = 0; s < 8; ++s)
                out[(size_t)r * cols * 8 + (size_t)c * 8 + s] = (int16_t)(((uint32_t)a[(size_t)r * cols + c] >> (4 * s)) & 15u);
}
/* inverse of unpack_i32_nibbles_first: codes u[K,N] (0..15) -> qweight[K/8,N] */
void orc_pack_i32_nibbles_first(const uint8_t *u, int K, int N, int32_t *out) {
    for (int r = 0; r < K / 8; ++r)
        for (int c = 0; c < N; ++c) {
            uint32_t w = 0;
            for (int s = 0; s < 8; ++s) w |= (uint32_t)(u[((size_t)r * 8 + s) * N + c] & 15u) << (4 * s);
            out[(size_t)r * N + c] = (int32_t)w;
        }
}
/* inverse of unpack_i32_nibbles_last: codes u[rows, cols] -> out[rows, cols/8] */
void orc_pack_i32_nibbles_last(const uint8_t *u, int rows, int cols, int32_t *out) {
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols / 8; ++c) {
            uint32_t w = 0;
            for (int s = 0; s < 8; ++s) w |= (uint32_t)(u[(size_t)r * cols + (size_t)c * 8 + s] & 15u) << (4 * s);
            out[(size_t)r * (cols / 8) + c] = (int32_t)w;
        }
}
/* pack_s4 + pack_b: kernels/esimd_dpas/dpas_s4_gptq.cpp:46-48,62-66
 * s4 b[K,N] -> u8 [K/2,N], low nibble = even k. */
void orc_pack_s4_along_k(const int8_t *b, int K, int N, uint8_t *out) {
    for (int kk = 0; kk < K; kk += 2)
        for (int j = 0; j < N; ++j)
            out[(size_t)(kk / 2) * N + j] = (uint8_t)(((uint8_t)b[(size_t)kk * N + j] & 0xF) |
                                                     (((uint8_t)b[(size_t)(kk + 1) * N + j] & 0xF) << 4));
}
/* pack_a: kernels/esimd_dpas/dpas_s4_gptq.cpp:55-60; s4 a[M,K] -> u8 [M,K/2] */
void orc_pack_s4_rows(const int8_t *a, int M, int K, uint8_t *out) {
    for (int i = 0; i < M; ++i)
        for (int kk = 0; kk < K; kk += 2)
            out[(size_t)i * (K / 2) + kk / 2] = (uint8_t)(((uint8_t)a[(size_t)i * K + kk] & 0xF) |
                                                         (((uint8_t)a[(size_t)i * K + kk + 1] & 0xF) << 4));
}

/* ------------------------------------------------------------------ */
/* integer / reference-formula GEMMs                                   */
/* ------------------------------------------------------------------ */
/* host_s32: kernels/nvfp4/bitcast_e2m1_s4.cpp:95-104 */
void orc_s32_gemm(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k) {
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            int32_t acc = 0;
            for (int kk = 0; kk < k; ++kk) acc += (int32_t)a[(size_t)i * k + kk] * (int32_t)b[(size_t)kk * n + j];
            c[(size_t)i * n + j] = acc;
        }
}

/* GPTQ s4 host oracle: kernels/esimd_dpas/dpas_s4_gptq_sc.cpp:273-288.
 * C[i,j] = half( sum_g float(s32_g) * a_s[i] * float(s[g,j]) ), s32_g exact. */
void orc_gptq_s4a_gemm(const int8_t *a, const float *a_scale, const int8_t *b,
                       const uint16_t *s_f16, int m, int n, int k, int gs, uint16_t *c_f16) {
    int ngrp = k / gs;
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            float acc = 0.f;
            for (int g = 0; g < ngrp; ++g) {
                int32_t s32 = 0;
                for (int kk = 0; kk < gs; ++kk) {
                    int ki = g * gs + kk;
                    s32 += (int32_t)a[(size_t)i * k + ki] * (int32_t)b[(size_t)ki * n + j];
                }
                acc += (float)s32 * a_scale[i] * orc_f16_to_f32(s_f16[(size_t)g * n + j]);
            }
            c_f16[(size_t)i * n + j] = orc_f32_to_f16(acc);
        }
}

/* NVFP4 LUT host oracle: kernels/nvfp4/nibble_lut_sc.cpp:319-330 (unpack_host :85-92).
 * C[i,j] = half( (sum_k float(a[i,k]) * float(q[k,j])) * a_s[i] * b_s[j] ). */
void orc_nvfp4_lut_gemm_s8a(const int8_t *a, const uint8_t *packed, const float *a_s,
                            const float *b_s, int m, int n, int k, uint16_t *c_f16) {
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            float acc = 0.f;
            for (int kk = 0; kk < k; ++kk) {
                uint8_t p = packed[(size_t)(kk / 2) * n + j];
                int8_t q = orc_e2m1_q((kk & 1) ? (uint8_t)(p >> 4) : (uint8_t)(p & 15));
                acc += (float)a[(size_t)i * k + kk] * (float)q;
            }
            c_f16[(size_t)i * n + j] = orc_f32_to_f16(acc * a_s[i] * b_s[j]);
        }
}

/* ------------------------------------------------------------------ */
/* W4A16 GPTQ                                                          */
/* ------------------------------------------------------------------ */
static inline int gptq_code(const int32_t *qweight, int N, int k, int n) {
    return (int)(((uint32_t)qweight[(size_t)(k >> 3) * N + n] >> (4 * (k & 7))) & 15u);
}
static inline int gptq_zero(const int32_t *qzeros, int N, int g, int n, int zero_offset) {
    if (!qzeros) return 8; /* symmetric: stored 7 + 1 (gptq_s4_dump.py:114, u - 8) */
    return (int)(((uint32_t)qzeros[(size_t)g * (N / 8) + (n >> 3)] >> (4 * (n & 7))) & 15u) + zero_offset;
}

/* w[k,n] = float(scales[g,n]) * (q[k,n] - zero_eff[g,n]); g = g_idx ? g_idx[k] : k/gs.
 * Layouts: gptq_s4_dump.py:106-114 (qweight [K/8,N] along K, qzeros [K/gs,N/8] along N).
 * The product of a 5-bit integer and an fp16 value is exact in fp32. */
void orc_gptq_dequant(const int32_t *qweight, const int32_t *qzeros,
                      const uint16_t *scales_f16, const int32_t *g_idx, int K, int N,
                      int group_size, int zero_offset, float *w) {
    for (int k = 0; k < K; ++k) {
        int g = g_idx ? g_idx[k] : k / group_size;
        for (int n = 0; n < N; ++n) {
            int d = gptq_code(qweight, N, k, n) - gptq_zero(qzeros, N, g, n, zero_offset);
            w[(size_t)k * N + n] = (float)d * orc_f16_to_f32(scales_f16[(size_t)g * N + n]);
        }
    }
}

/* W4A16 restatement of the group-partial loop of dpas_s4_gptq_sc.cpp:273-288 with
 * real-valued activations:
 *   part_g = sum_{k in g, ascending} a[m,k] * (q[k,n] - z[g,n])      (fp32)
 *   c[m,n] = sum_{g ascending} part_g * s[g,n]                      (fp32)
 * With g_idx, group g holds the k with g_idx[k] == g (act_order).
 * Vectorised across n only, so each output sees exactly the scalar loop order. */
#define ORC_NB 256
void orc_gptq_gemm(const float *a, const int32_t *qweight, const int32_t *qzeros,
                   const uint16_t *scales_f16, const int32_t *g_idx, int M, int N, int K,
                   int group_size, int zero_offset, float *c, int threads) {
    int ngrp = K / group_size;
    int nblocks = (N + ORC_NB - 1) / ORC_NB;
    set_threads(threads);
#pragma omp parallel
    {
        float *part = (float *)malloc(sizeof(float) * (size_t)ngrp * ORC_NB);
        float acc[ORC_NB];
        float z[ORC_NB];
#pragma omp for collapse(2) schedule(dynamic, 1)
        for (int m = 0; m < M; ++m)
            for (int nb = 0; nb < nblocks; ++nb) {
                int n0 = nb * ORC_NB, nw = N - n0 < ORC_NB ? N - n0 : ORC_NB;
                memset(part, 0, sizeof(float) * (size_t)ngrp * ORC_NB);
                for (int k = 0; k < K; ++k) {
                    int g = g_idx ? g_idx[k] : k / group_size;
                    float av = a[(size_t)m * K + k];
                    float *pg = part + (size_t)g * ORC_NB;
                    const int32_t *qrow = qweight + (size_t)(k >> 3) * N + n0;
                    int sh = 4 * (k & 7);
                    for (int j = 0; j < nw; ++j) z[j] = (float)gptq_zero(qzeros, N, g, n0 + j, zero_offset);
                    for (int j = 0; j < nw; ++j) {
                        float d = (float)(((uint32_t)qrow[j] >> sh) & 15u) - z[j];
                        pg[j] += av * d;
                    }
                }
                for (int j = 0; j < nw; ++j) acc[j] = 0.f;
                for (int g = 0; g < ngrp; ++g) {
                    const uint16_t *srow = scales_f16 + (size_t)g * N + n0;
                    const float *pg = part + (size_t)g * ORC_NB;
                    for (int j = 0; j < nw; ++j) acc[j] += pg[j] * orc_f16_to_f32(srow[j]);
                }
                for (int j = 0; j < nw; ++j) c[(size_t)m * N + n0 + j] = acc[j];
            }
        free(part);
    }
}

/* act_order load-time permutation: perm = stable argsort(g_idx).  Row j of the
 * repacked weight is row perm[j] of the checkpoint, so groups become contiguous. */
void orc_gptq_act_order_perm(const int32_t *g_idx, int K, int group_size, int32_t *perm) {
    int ngrp = K / group_size;
    int *count = (int *)calloc((size_t)ngrp + 1, sizeof(int));
    for (int k = 0; k < K; ++k) count[g_idx[k] + 1]++;
    for (int g = 0; g < ngrp; ++g) count[g + 1] += count[g];
    for (int k = 0; k < K; ++k) perm[count[g_idx[k]]++] = k;
    free(count);
}

/* ------------------------------------------------------------------ */
/* NVFP4                                                               */
/* ------------------------------------------------------------------ */
static inline uint8_t nvfp4_nib(const uint8_t *w, int layout, int K, int N, int k, int n) {
    uint8_t p = (layout == ORC_NVFP4_KN) ? w[(size_t)(k >> 1) * N + n] : w[(size_t)n * (K / 2) + (k >> 1)];
    return (k & 1) ? (uint8_t)(p >> 4) : (uint8_t)(p & 15);
}
static inline float nvfp4_block_scale(const uint8_t *scale, int kind, int N, int k, int n) {
    size_t i = (size_t)(k >> 4) * N + n;
    if (kind == ORC_SCALE_E4M3) return orc_e4m3_value(scale[i]);
    uint16_t h; memcpy(&h, scale + 2 * i, 2);
    return orc_bf16_to_f32(h);
}

/* w[k,n] = (e2m1(nib[k,n]) * scale[k/16,n]) * global.  Packing: nibble_lut_sc.cpp:77-92
 * (two nibbles per byte along K, low = even k); block scales: one per 16 K
 * (g16_scale_landmine.py:49-57); format: nvfp4-vs-ocp-mx.md:9-60. */
void orc_nvfp4_dequant(const uint8_t *w, int layout, const uint8_t *scale, int scale_kind,
                       float global_scale, int K, int N, float *out) {
    for (int k = 0; k < K; ++k)
        for (int n = 0; n < N; ++n) {
            float v = orc_e2m1_value(nvfp4_nib(w, layout, K, N, k, n)) * nvfp4_block_scale(scale, scale_kind, N, k, n);
            out[(size_t)k * N + n] = v * global_scale;
        }
}

/* NVFP4 W4A16 restatement of nibble_lut_sc.cpp:319-330 with E4M3 block scales and
 * the fp32 tensor scale: acc = sum_k a[m,k] * (e2m1 * s_blk)  (fp32, k ascending);
 * c = acc * global. */
void orc_nvfp4_gemm(const float *a, const uint8_t *w, int layout, const uint8_t *scale,
                    int scale_kind, float global_scale, int M, int N, int K, float *c,
                    int threads) {
    int nblocks = (N + ORC_NB - 1) / ORC_NB;
    set_threads(threads);
#pragma omp parallel
    {
        float acc[ORC_NB];
#pragma omp for collapse(2) schedule(dynamic, 1)
        for (int m = 0; m < M; ++m)
            for (int nb = 0; nb < nblocks; ++nb) {
                int n0 = nb * ORC_NB, nw = N - n0 < ORC_NB ? N - n0 : ORC_NB;
                for (int j = 0; j < nw; ++j) acc[j] = 0.f;
                for (int k = 0; k < K; ++k) {
                    float av = a[(size_t)m * K + k];
                    for (int j = 0; j < nw; ++j) {
                        float wv = orc_e2m1_value(nvfp4_nib(w, layout, K, N, k, n0 + j)) *
                                   nvfp4_block_scale(scale, scale_kind, N, k, n0 + j);
                        acc[j] += av * wv;
                    }
                }
                for (int j = 0; j < nw; ++j) c[(size_t)m * N + n0 + j] = acc[j] * global_scale;
            }
    }
}

/* NVFP4 activation quantiser (two-level scaling, nvfp4-vs-ocp-mx.md:9-18):
 * per row m and 16-element block b:
 *   amax  = max |a|;  sf = e4m3_rne(amax / (6 * global_dec));
 *   sdec  = e4m3(sf) * global_dec;  code = e2m1_rne(a / sdec)  (0 when sdec == 0).
 * codes [M, K/2] (low nibble = even k), sf [M, K/16]. */
void orc_nvfp4_quant_act(const float *a, int M, int K, float global_dec, uint8_t *codes,
                         uint8_t *sf) {
    float denom6 = 6.0f * global_dec;
    for (int m = 0; m < M; ++m)
        for (int b = 0; b < K / 16; ++b) {
            const float *x = a + (size_t)m * K + (size_t)b * 16;
            float amax = 0.f;
            for (int i = 0; i < 16; ++i) { float v = fabsf(x[i]); if (v > amax) amax = v; }
            uint8_t s = orc_e4m3_from_f32(amax / denom6);
            float sdec = orc_e4m3_value(s) * global_dec;
            /* one correctly rounded reciprocal per block, then a product per element */
            float inv = sdec != 0.f ? 1.0f / sdec : 0.f;
            sf[(size_t)m * (K / 16) + b] = s;
            for (int i = 0; i < 16; i += 2) {
                uint8_t lo = sdec != 0.f ? orc_e2m1_from_f32(x[i] * inv) : 0;
                uint8_t hi = sdec != 0.f ? orc_e2m1_from_f32(x[i + 1] * inv) : 0;
                codes[(size_t)m * (K / 2) + (size_t)b * 8 + i / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
}

void orc_nvfp4_act_dequant(const uint8_t *codes, const uint8_t *sf, float global_dec,
                           int M, int K, float *out) {
    for (int m = 0; m < M; ++m)
        for (int k = 0; k < K; ++k) {
            uint8_t p = codes[(size_t)m * (K / 2) + k / 2];
            uint8_t nib = (k & 1) ? (uint8_t)(p >> 4) : (uint8_t)(p & 15);
            float v = orc_e2m1_value(nib) * orc_e4m3_value(sf[(size_t)m * (K / 16) + k / 16]);
            out[(size_t)m * K + k] = v * global_dec;
        }
}

/* ------------------------------------------------------------------ */
/* epilogue quant                                                      */
/* ------------------------------------------------------------------ */
/* quant_one + host_rmsnorm_quant: kernels/epilogue_quant/rmsnorm_epilogue.cpp:39-70 */
static int8_t quant_one(float y, float scale) {
    float q = scale > 0.f ? y / scale : 0.f;
    q = nearbyintf(q);
    if (q > 127.f) q = 127.f;
    if (q < -127.f) q = -127.f;
    return (int8_t)q;
}

void orc_rmsnorm_quant_s8(const float *x, int8_t *q, float *scale, int m, int k, float eps) {
    for (int i = 0; i < m; ++i) {
        const float *row = x + (size_t)i * k;
        float ss = 0.f;
        for (int j = 0; j < k; ++j) ss += row[j] * row[j];
        float inv = 1.f / sqrtf(ss / (float)k + eps);
        float amax = 0.f;
        for (int j = 0; j < k; ++j) {
            float y = row[j] * inv;
            float ay = y < 0.f ? -y : y;
            if (ay > amax) amax = ay;
        }
        float s = amax / 127.f;
        if (s <= 0.f) s = 1.f;
        scale[i] = s;
        for (int j = 0; j < k; ++j) q[(size_t)i * k + j] = quant_one(row[j] * inv, s);
    }
}

/* RMSNorm -> NVFP4 activations (the fused producer of the NVFP4 GEMM): the
 * normalisation of rmsnorm_epilogue.cpp:49-56 (sequential fp32 sum of squares,
 * inv = 1 / sqrt(ss / k + eps)), y = bf16(x * inv [* gamma]) rounded once, then
 * orc_nvfp4_quant_act on the row.  codes [m, k/2], sf [m, k/16] row-major. */
void orc_rmsnorm_nvfp4(const float *x, const float *gamma, int m, int k, float eps, float global_dec,
                       uint8_t *codes, uint8_t *sf) {
    float *y = (float *)malloc((size_t)k * sizeof(float));
    if (!y) return;
    for (int i = 0; i < m; ++i) {
        const float *row = x + (size_t)i * k;
        float ss = 0.f;
        for (int j = 0; j < k; ++j) ss += row[j] * row[j];
        const float inv = 1.f / sqrtf(ss / (float)k + eps);
        for (int j = 0; j < k; ++j) {
            float v = row[j] * inv;
            if (gamma) v = v * gamma[j];
            y[j] = orc_bf16_to_f32(orc_f32_to_bf16(v));
        }
        orc_nvfp4_quant_act(y, 1, k, global_dec, codes + (size_t)i * (k / 2), sf + (size_t)i * (k / 16));
    }
    free(y);
}

/* fp8-E4M3 per-row cast: the same absmax contract as rmsnorm_epilogue.cpp:56-69 with
 * qmax 448 (E4M3 max finite): s = amax/448 (1 if 0); q = e4m3_rne_satfinite(y / s). */
void orc_rowscale_fp8(const float *y, int M, int N, uint8_t *q, float *scale) {
    for (int i = 0; i < M; ++i) {
        const float *row = y + (size_t)i * N;
        float amax = 0.f;
        for (int j = 0; j < N; ++j) { float a = fabsf(row[j]); if (a > amax) amax = a; }
        float s = amax / 448.f;
        if (s <= 0.f) s = 1.f;
        scale[i] = s;
        for (int j = 0; j < N; ++j) q[(size_t)i * N + j] = orc_e4m3_from_f32(row[j] / s);
    }
}

/* ------------------------------------------------------------------ */
/* metrics: dpas_s4_gptq_sc.cpp:312-327                                 */
/* ------------------------------------------------------------------ */
double orc_cosine(const float *x, const float *y, size_t n) {
    double dot = 0, na = 0, nb = 0;
    for (size_t i = 0; i < n; ++i) {
        dot += (double)x[i] * y[i];
        na += (double)x[i] * x[i];
        nb += (double)y[i] * y[i];
    }
    return (na > 0 && nb > 0) ? dot / sqrt(na * nb) : 0.0;
}
double orc_max_abs(const float *x, const float *y, size_t n) {
    double mx = 0;
    for (size_t i = 0; i < n; ++i) {
        double d = fabs((double)x[i] - (double)y[i]);
        if (d > mx) mx = d;
    }
    return mx;
}
double orc_rel_frob(const float *got, const float *ref, size_t n) {
    double num = 0, den = 0;
    for (size_t i = 0; i < n; ++i) {
        double d = (double)got[i] - ref[i];
        num += d * d;
        den += (double)ref[i] * ref[i];
    }
    return den > 0 ? sqrt(num / den) : sqrt(num);
}
