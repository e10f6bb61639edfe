// w4_common.cuh -- shared helpers for libw4 (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include <cooperative_groups.h>

#include "w4.h"  // include/ is on the include path

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libw4 targets sm_100a only"
#endif

namespace w4 {

// ---- error reporting (thread-local one-line reason) ----
void set_error(const char *fmt, ...);
const char *last_error();

#define W4_REQUIRE(cond, code, ...)        \
    do {                                   \
        if (!(cond)) {                     \
            ::w4::set_error(__VA_ARGS__);  \
            return (code);                 \
        }                                  \
    } while (0)

#define W4_CUDA_TRY(expr)                                                             \
    do {                                                                              \
        cudaError_t _e = (expr);                                                      \
        if (_e != cudaSuccess) {                                                      \
            ::w4::set_error("%s: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, \
                            __LINE__);                                                \
            return W4_ERR_CUDA;                                                       \
        }                                                                             \
    } while (0)

#define W4_LAUNCH_CHECK()                                                                   \
    do {                                                                                    \
        cudaError_t _e = cudaGetLastError();                                                \
        if (_e != cudaSuccess) {                                                            \
            ::w4::set_error("kernel launch: %s (%s:%d)", cudaGetErrorString(_e), __FILE__, \
                            __LINE__);                                                      \
            return W4_ERR_CUDA;                                                             \
        }                                                                                   \
    } while (0)

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int num_sms();
int launch_overlap();  // the process-wide W4_OVERLAP_* mode (w4_set_launch_overlap)

// ---- device helpers ----
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;  // (a & b) | c
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ld_nc_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2::evict_normal [%0];" ::"l"(p));
}

// 16-byte asynchronous global -> shared copy (L2 only), in commit groups.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
template <int BYTES>  // 4 or 8 (L1-allocating form; 16 uses cp_async16)
__device__ __forceinline__ void cp_async_small(void *smem, const void *gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(s), "l"(gmem), "n"(BYTES) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// D = A(16x16, row) * B(16x8, col) + C, fp32 accumulate.  Legacy warp MMA;
// used by the decode kernels whose bound is HBM, not the tensor pipe.
template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma_16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1,
                                                         uint32_t a2, uint32_t a3, uint32_t b0,
                                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma_16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1,
                                                  uint32_t a2, uint32_t a3, uint32_t b0,
                                                  uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename T> struct Conv;
template <> struct Conv<__half> {
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
    // a packed pair (low half first) -> floats
    static __device__ __forceinline__ float2 to_f2(uint32_t w) {
        return __half22float2(*reinterpret_cast<const __half2 *>(&w));
    }
};
template <> struct Conv<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
    static __device__ __forceinline__ float2 to_f2(uint32_t w) {
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    }
};

__device__ __forceinline__ float f16_bits_to_f(uint16_t b) {
    return __half2float(__ushort_as_half(b));
}

// Sum (or max) of v over the CTA, returned to every thread; sh holds 32 floats.
__device__ __forceinline__ float block_reduce(float v, bool is_max, float *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, u) : v + u;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    v = lane < (blockDim.x >> 5) ? sh[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, u) : v + u;
    }
    return v;  // every thread holds the result
}

// e4m3fn -> f32 (exact; 0x7F/0xFF decode to NaN).
__device__ __forceinline__ float e4m3_to_f(uint32_t b) {
    uint32_t e = (b >> 3) & 0xF, m = b & 7;
    float v;
    if (e == 0) {
        v = __int2float_rn(m) * 0.001953125f;
    } else {
        v = __uint_as_float(((e + 120u) << 23) | (m << 20));
        if (e == 15 && m == 7) v = __int_as_float(0x7fc00000);
    }
    return (b & 0x80) ? -v : v;
}

// f32 -> e4m3fn, round-to-nearest-even, saturating to +-448 (NaN -> 0x7F).
__device__ __forceinline__ uint32_t f_to_e4m3(float x) {
    uint32_t u = __float_as_uint(x);
    uint32_t s = (u >> 24) & 0x80;
    uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return 0x7F;
    if (a >= 0x43E00000u) return s | 0x7E;
    if (a < 0x3C800000u) {
        float q = rintf(__uint_as_float(a) * 512.0f);
        return s | (uint32_t)q;
    }
    int e = (int)(a >> 23) - 127;
    uint32_t m = a & 0x7FFFFFu;
    uint32_t q = m >> 20, rem = m & 0xFFFFFu;
    if (rem > 0x80000u || (rem == 0x80000u && (q & 1))) q++;
    uint32_t code = ((uint32_t)(e + 7) << 3) + q;
    if (code > 0x7E) code = 0x7E;
    return s | code;
}

// f32 -> e2m1 code (RNE, saturating to +-6).
__device__ __forceinline__ uint32_t f_to_e2m1(float x) {
    uint32_t s = (__float_as_uint(x) >> 31) ? 8u : 0u;
    float a = fabsf(x);
    uint32_t c;
    if (a <= 0.25f) c = 0;
    else if (a < 0.75f) c = 1;
    else if (a <= 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a <= 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a <= 5.0f) c = 6;
    else c = 7;
    return s | c;
}

__device__ __forceinline__ float e2m1_to_f(uint32_t nib) {
    // magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}
    const uint32_t e = (nib >> 1) & 3, m = nib & 1;
    float v = (e == 0) ? 0.5f * (float)m : __uint_as_float(((e + 126u) << 23) | (m << 22));
    return (nib & 8) ? -v : v;
}

// ---- split-K reduction of per-lane accumulators ----
// The WARPS warps of a CTA each hold NE floats per lane for the same output
// tile (different k ranges).  They are summed through shared memory; when the
// kernel runs as a thread-block cluster of `ks` CTAs along K, the leader CTA
// (cluster rank 0) adds the other CTAs' sums over distributed shared memory.
// Every thread of every CTA must call this exactly once.  Returns the summed
// tile (index e*32 + lane) in the leader and nullptr elsewhere.
template <int NE, int WARPS> struct SplitKSmem {
    float red[WARPS][NE][32];
    float part[NE * 32];
};

template <int NE, int WARPS>
__device__ __forceinline__ const float *splitk_reduce(SplitKSmem<NE, WARPS> &sm,
                                                      const float (&acc)[NE], int ks) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int e = 0; e < NE; ++e) sm.red[warp][e][lane] = acc[e];
    __syncthreads();
    for (int idx = threadIdx.x; idx < NE * 32; idx += blockDim.x) {
        const int e = idx >> 5, l = idx & 31;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) v += sm.red[w][e][l];
        sm.part[idx] = v;
    }
    if (ks <= 1) {
        __syncthreads();
        return sm.part;
    }
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const bool leader = cluster.block_rank() == 0;
    if (leader) {
        for (int idx = threadIdx.x; idx < NE * 32; idx += blockDim.x) {
            float v = sm.part[idx];
            for (int r = 1; r < ks; ++r) v += cluster.map_shared_rank(sm.part, r)[idx];
            (&sm.red[0][0][0])[idx] = v;
        }
    }
    cluster.sync();  // remote reads done before any CTA of the cluster exits
    return leader ? &sm.red[0][0][0] : nullptr;
}

__device__ __forceinline__ void store_out(void *C, int c_dtype, size_t o, float v) {
    if (c_dtype == W4_F32) reinterpret_cast<float *>(C)[o] = v;
    else if (c_dtype == W4_BF16) reinterpret_cast<__nv_bfloat16 *>(C)[o] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half *>(C)[o] = __float2half_rn(v);
}

}  // namespace w4
