// epilogue.cu -- epilogue_quant kernels for sm_100a.
//
// rmsnorm_quant_s8 restates the contract of the reference's fused kernel
// (kernels/epilogue_quant/rmsnorm_epilogue.cpp:118-151, host oracle :39-70):
// one CTA per row instead of one work-item per row, 128-bit loads, warp-shuffle
// reductions.  Everything after the sum of squares uses the host's operation
// order with IEEE division / square root, so codes can differ from the host
// only where the parallel sum of squares rounds differently (|dq| <= 1, the
// reference's own acceptance bound, rmsnorm_epilogue.cpp:193-204).
#include "tma_util.cuh"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

constexpr int kRowThreads = 256;

__device__ __forceinline__ int8_t quant_s8(float y, float s) {
    float q = rintf(__fdiv_rn(y, s));
    q = fminf(fmaxf(q, -127.f), 127.f);
    return (int8_t)q;
}

__global__ void __launch_bounds__(kRowThreads)
rmsnorm_quant_s8_kernel(const uint16_t *__restrict__ x, int8_t *__restrict__ q,
                        float *__restrict__ scale, int K, float eps) {
    __shared__ float sh[32];
    const int row = blockIdx.x;
    const uint16_t *xr = x + (size_t)row * K;
    int8_t *qr = q + (size_t)row * K;
    const int nvec = K / 8;  // K % 8 == 0 is validated by the caller

    float ss = 0.f;
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        const uint4 u = ld_nc_v4(xr + (size_t)v * 8);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            ss += f.x * f.x + f.y * f.y;
        }
    }
    ss = block_reduce(ss, false, sh);
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));

    float amax = 0.f;
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        const uint4 u = ld_nc_v4(xr + (size_t)v * 8);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            amax = fmaxf(amax, fmaxf(fabsf(__fmul_rn(f.x, inv)), fabsf(__fmul_rn(f.y, inv))));
        }
    }
    amax = block_reduce(amax, true, sh);
    float s = __fdiv_rn(amax, 127.f);
    if (s <= 0.f) s = 1.f;
    if (threadIdx.x == 0) scale[row] = s;

    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        const uint4 u = ld_nc_v4(xr + (size_t)v * 8);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
        uint32_t out[2] = {0, 0};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            const uint32_t lo = (uint8_t)quant_s8(__fmul_rn(f.x, inv), s);
            const uint32_t hi = (uint8_t)quant_s8(__fmul_rn(f.y, inv), s);
            out[i >> 1] |= (lo | (hi << 8)) << (16 * (i & 1));
        }
        *reinterpret_cast<uint2 *>(qr + (size_t)v * 8) = make_uint2(out[0], out[1]);
    }
}

int rmsnorm_quant_s8(const uint16_t *x, int8_t *q, float *scale, int M, int K, float eps,
                     cudaStream_t st) {
    rmsnorm_quant_s8_kernel<<<M, kRowThreads, 0, st>>>(x, q, scale, K, eps);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

// ---- per-row fp8-E4M3 cast: s = max|y|/448 (1 if 0), q = e4m3(y / s) ----
template <typename T>
__device__ __forceinline__ float load_as_f(const void *p, size_t i) {
    if constexpr (sizeof(T) == 4) return reinterpret_cast<const float *>(p)[i];
    else return Conv<T>::to_f(reinterpret_cast<const T *>(p)[i]);
}

template <typename T>
__global__ void __launch_bounds__(kRowThreads)
rowscale_fp8_kernel(const void *__restrict__ y, uint8_t *__restrict__ q,
                    float *__restrict__ row_scale, int N) {
    __shared__ float sh[32];
    const int row = blockIdx.x;
    const size_t base = (size_t)row * N;
    float amax = 0.f;
    for (int j = threadIdx.x; j < N; j += blockDim.x) amax = fmaxf(amax, fabsf(load_as_f<T>(y, base + j)));
    amax = block_reduce(amax, true, sh);
    float s = __fdiv_rn(amax, 448.f);
    if (s <= 0.f) s = 1.f;
    if (threadIdx.x == 0) row_scale[row] = s;
    for (int j = threadIdx.x; j < N; j += blockDim.x)
        q[base + j] = (uint8_t)f_to_e4m3(__fdiv_rn(load_as_f<T>(y, base + j), s));
}

// The cast when a decode GEMM has already folded the row maxima of |y| into rowmax (fp32 bits):
// CTA (chunk, row) casts 8 values per thread of its 2048-value chunk, with the row's scale
// computed as above; chunk 0 stores it.  Each CTA counts itself on rowcnt[row] after reading
// the maximum (acquire-release), and the last one zeroes rowmax[row] for the next call (the
// counter wraps to zero).
constexpr int kCastChunk = 8 * kRowThreads;
__global__ void __launch_bounds__(kRowThreads)
rowscale_fp8_amax_kernel(const float *__restrict__ y, unsigned int *__restrict__ rowmax,
                         unsigned int *__restrict__ rowcnt, uint8_t *__restrict__ q,
                         float *__restrict__ row_scale, int N) {
    __shared__ float s_sh;
    const int row = blockIdx.y;
    if (threadIdx.x == 0) {
        const float amax = __uint_as_float(*reinterpret_cast<volatile unsigned int *>(&rowmax[row]));
        float s = __fdiv_rn(amax, 448.f);
        if (s <= 0.f) s = 1.f;
        s_sh = s;
        if (blockIdx.x == 0) row_scale[row] = s;
        if (atom_inc_acq_rel(&rowcnt[row], gridDim.x - 1) == gridDim.x - 1) rowmax[row] = 0u;
    }
    __syncthreads();
    const float s = s_sh;
    const int j = blockIdx.x * kCastChunk + threadIdx.x * 8;
    if (j >= N) return;
    const float4 a = __ldcs(reinterpret_cast<const float4 *>(y + (size_t)row * N + j));
    const float4 b = __ldcs(reinterpret_cast<const float4 *>(y + (size_t)row * N + j + 4));
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i >> 2] |= f_to_e4m3(__fdiv_rn(v[i], s)) << (8 * (i & 3));
    *reinterpret_cast<uint2 *>(q + (size_t)row * N + j) = make_uint2(w[0], w[1]);
}

int rowscale_fp8_amax(const float *y, unsigned int *rowmax, unsigned int *rowcnt, uint8_t *q, float *row_scale,
                      int M, int N, cudaStream_t st) {
    if (M > 16 || N % 8 || !aligned(y, 16) || !aligned(q, 8)) return -1;
    const dim3 grid((N + kCastChunk - 1) / kCastChunk, M);
    rowscale_fp8_amax_kernel<<<grid, kRowThreads, 0, st>>>(y, rowmax, rowcnt, q, row_scale, N);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

int rowscale_fp8(const void *y, int y_dtype, uint8_t *q, float *row_scale, int M, int N,
                 cudaStream_t st) {
    if (y_dtype == W4_F32) rowscale_fp8_kernel<float><<<M, kRowThreads, 0, st>>>(y, q, row_scale, N);
    else if (y_dtype == W4_BF16) rowscale_fp8_kernel<__nv_bfloat16><<<M, kRowThreads, 0, st>>>(y, q, row_scale, N);
    else rowscale_fp8_kernel<__half><<<M, kRowThreads, 0, st>>>(y, q, row_scale, N);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

}  // namespace w4
