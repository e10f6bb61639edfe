// nvfp4.cu -- NVFP4 (E2M1 nibbles, one E4M3 scale per 16 K, fp32 tensor scale)
// kernels for sm_100a.
//
// Packing (kernels/nvfp4/nibble_lut_sc.cpp:77-92 of the reference): two codes per
// byte along K, low nibble = even k.  Two layouts: KN = u8 [K/2, N] (the
// reference kernel's own) and NK = u8 [N, K/2] (the external operator's w with
// stride(0)==1, kernels/nvfp4/bench_nvfp4_m1.py:58-61).  Block scales are
// [K/16, N] in both.
#include <cooperative_groups.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include <mutex>

#include "nvfp4_util.cuh"
#include "tma_util.cuh"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace cg = cooperative_groups;

namespace w4 {

__device__ __forceinline__ uint32_t nib_at(const uint8_t *w, int layout, int K, int N, int k,
                                           int n) {
    const uint8_t p = (layout == W4_NVFP4_KN) ? w[(size_t)(k >> 1) * N + n]
                                              : w[(size_t)n * (K / 2) + (k >> 1)];
    return (k & 1) ? (uint32_t)(p >> 4) : (uint32_t)(p & 15);
}

__device__ __forceinline__ float block_scale_f(const void *scale, int scale_dtype, int N, int k,
                                               int n) {
    const size_t i = (size_t)(k >> 4) * N + n;
    if (scale_dtype == W4_E4M3) return e4m3_to_f(reinterpret_cast<const uint8_t *>(scale)[i]);
    return __bfloat162float(__ushort_as_bfloat16(reinterpret_cast<const uint16_t *>(scale)[i]));
}

// ---- dequant (bit-exact): out[k,n] = (e2m1 * s) * global ----
__global__ void nvfp4_dequant_kernel(const uint8_t *__restrict__ w, int layout,
                                     const void *__restrict__ scale, int scale_dtype,
                                     const float *__restrict__ global_scale, int K, int N,
                                     float *__restrict__ out) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int k = blockIdx.y;
    if (n >= N) return;
    const float g = global_scale ? *global_scale : 1.0f;
    const float v = __fmul_rn(e2m1_to_f(nib_at(w, layout, K, N, k, n)),
                              block_scale_f(scale, scale_dtype, N, k, n));
    out[(size_t)k * N + n] = __fmul_rn(v, g);
}

int nvfp4_dequant(const uint8_t *w, int layout, const void *scale, int scale_dtype,
                  const float *global_scale, int K, int N, float *out, cudaStream_t st) {
    dim3 block(256), grid((N + 255) / 256, K);
    nvfp4_dequant_kernel<<<grid, block, 0, st>>>(w, layout, scale, scale_dtype, global_scale, K,
                                                 N, out);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

// ---- activation quantiser: one thread per 16-element block ----
// sf = e4m3(amax / (6 g)), d = e4m3(sf) * g, code = e2m1(a * (1/d)) with one
// correctly rounded reciprocal per block.  ATOMS: the scales go straight into
// the 512-byte atom layout of the block-scaled GEMM (rows padded to 128 with
// zero scales), else row-major [M, K/16].
// Byte offset of block scale (row m, 16-k block kb) in the row-major [rows, nb]
// layout, or in the 512-byte atoms of the block-scaled GEMM (128 rows x 4 blocks).
template <bool ATOMS> __device__ __forceinline__ size_t sf_offset(int m, int kb, int nb) {
    if constexpr (ATOMS)
        return ((size_t)(m >> 7) * (nb >> 2) + (kb >> 2)) * 512 + (m & 31) * 16 + ((m >> 5) & 3) * 4 + (kb & 3);
    else
        return (size_t)m * nb + kb;
}

// One 16-value block: the UE4M3 scale byte and the 16 E2M1 codes (8 bytes, low
// nibble = even k).  v holds values exactly representable in bf16.
__device__ __forceinline__ uint32_t nvfp4_block(const float (&v)[16], float g, uint2 &codes) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    // hardware conversions (one instruction each): f32 -> e4m3 rounds to nearest
    // even and saturates at 448 like f_to_e4m3 (amax is never NaN here); e4m3 ->
    // f16 is exact
    const uint32_t s = (uint32_t)__nv_cvt_float_to_fp8(__fdiv_rn(amax, __fmul_rn(6.0f, g)), __NV_SATFINITE, __NV_E4M3);
    const float sdec = __fmul_rn(__half2float(__ushort_as_half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)s, __NV_E4M3).x)), g);
    const float inv = sdec != 0.f ? __frcp_rn(sdec) : 0.f;
    // hardware E2M1 conversion: round to nearest even, saturating at +-6 (the
    // rounding rule of f_to_e2m1 / the host quantiser)
    uint32_t packed[2] = {0, 0};
    if (sdec != 0.f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t c2 = __nv_cvt_float2_to_fp4x2(make_float2(__fmul_rn(v[2 * i], inv), __fmul_rn(v[2 * i + 1], inv)),
                                                         __NV_E2M1, cudaRoundNearest);
            packed[i >> 2] |= (c2 & 0xFFu) << (8 * (i & 3));
        }
    }
    codes = make_uint2(packed[0], packed[1]);
    return s;
}

template <bool ATOMS>
__global__ void nvfp4_quant_act_kernel(const uint16_t *__restrict__ a, int M, int K,
                                       const float *__restrict__ a_global,
                                       uint8_t *__restrict__ codes, uint8_t *__restrict__ sf, int rows) {
    const long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int nb = K / 16;
    if (b >= (long)rows * nb) return;
    const int m = (int)(b / nb), kb = (int)(b % nb);
    const size_t si = sf_offset<ATOMS>(m, kb, nb);
    if (m >= M) {  // padding row of the last tile
        sf[si] = 0;
        return;
    }
    const uint16_t *x = a + (size_t)m * K + (size_t)kb * 16;
    const uint4 u0 = ld_nc_v4(x), u1 = ld_nc_v4(x + 8);
    const uint32_t wv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    float v[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[2 * i] = __uint_as_float(wv[i] << 16);
        v[2 * i + 1] = __uint_as_float(wv[i] & 0xFFFF0000u);
    }
    uint2 q;
    sf[si] = (uint8_t)nvfp4_block(v, *a_global, q);
    *reinterpret_cast<uint2 *>(codes + (size_t)m * (K / 2) + (size_t)kb * 8) = q;
}

// Fused producer (RMSNorm -> NVFP4 activations, one CTA per row):
//   inv = 1 / sqrt(sum(x^2) / K + eps)      (fp32 sum, IEEE divide / square root)
//   y   = bf16(x * inv [* gamma])           (one rounding to bf16 per value)
//   codes, scales = the 16-block quantisation of y (nvfp4_block), scales in the
//   atom layout the block-scaled GEMM reads; rows M..rows-1 (the last 128-row
//   tile's padding) get zero codes and zero scales.
// The normalisation is the reference's contract (rmsnorm_epilogue.cpp:39-56,
// without its s8 cast); the quantisation is w4_nvfp4_quant_act's, so the result
// equals quantising the bf16 RMSNorm output in a second pass.
// One 16-k block of the producer: y = bf16(x * inv [* gamma]), quantised.
template <typename T, bool GAMMA>
__device__ __forceinline__ void rmsnorm_nvfp4_block(const uint32_t (&wv)[8], const T *__restrict__ gamma, int kb,
                                                    float inv, float g, uint8_t *__restrict__ cr,
                                                    uint8_t *__restrict__ sf, int row, int nb) {
    uint32_t gv[8] = {};
    if constexpr (GAMMA) {
        const uint4 g0 = ld_nc_v4(gamma + (size_t)kb * 16), g1 = ld_nc_v4(gamma + (size_t)kb * 16 + 8);
        gv[0] = g0.x, gv[1] = g0.y, gv[2] = g0.z, gv[3] = g0.w;
        gv[4] = g1.x, gv[5] = g1.y, gv[6] = g1.z, gv[7] = g1.w;
    }
    float v[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float2 f = Conv<T>::to_f2(wv[i]);
        float y0 = __fmul_rn(f.x, inv), y1 = __fmul_rn(f.y, inv);
        if constexpr (GAMMA) {
            const float2 gg = Conv<T>::to_f2(gv[i]);
            y0 = __fmul_rn(y0, gg.x);
            y1 = __fmul_rn(y1, gg.y);
        }
        v[2 * i] = __bfloat162float(__float2bfloat16_rn(y0));
        v[2 * i + 1] = __bfloat162float(__float2bfloat16_rn(y1));
    }
    uint2 q;
    sf[sf_offset<true>(row, kb, nb)] = (uint8_t)nvfp4_block(v, g, q);
    *reinterpret_cast<uint2 *>(cr + (size_t)kb * 8) = q;
}

// BPT > 0: thread t holds 16-k blocks t, t + blockDim, ... (at most BPT) in
// registers, so x is read once; BPT == 0 (very wide rows): x is read twice.
template <typename T, bool GAMMA, int BPT>
__global__ void __launch_bounds__(256)
rmsnorm_nvfp4_kernel(const T *__restrict__ x, const T *__restrict__ gamma, float eps,
                     const float *__restrict__ a_global, uint8_t *__restrict__ codes, uint8_t *__restrict__ sf,
                     int M, int K) {
    __shared__ float sh[32];
    const int row = blockIdx.x, nb = K / 16;
    uint8_t *cr = codes + (size_t)row * (K / 2);
    if (row >= M) {
        for (int kb = threadIdx.x; kb < nb; kb += blockDim.x) {
            sf[sf_offset<true>(row, kb, nb)] = 0;
            *reinterpret_cast<uint2 *>(cr + (size_t)kb * 8) = make_uint2(0, 0);
        }
        return;
    }
    const T *xr = x + (size_t)row * K;
    float ss = 0.f;
    uint32_t xw[BPT > 0 ? BPT : 1][8];
    if constexpr (BPT > 0) {
#pragma unroll
        for (int i = 0; i < BPT; ++i) {
            const int kb = threadIdx.x + i * blockDim.x;
            uint4 u0 = make_uint4(0, 0, 0, 0), u1 = u0;
            if (kb < nb) {
                u0 = ld_nc_v4(xr + (size_t)kb * 16);
                u1 = ld_nc_v4(xr + (size_t)kb * 16 + 8);
            }
            xw[i][0] = u0.x, xw[i][1] = u0.y, xw[i][2] = u0.z, xw[i][3] = u0.w;
            xw[i][4] = u1.x, xw[i][5] = u1.y, xw[i][6] = u1.z, xw[i][7] = u1.w;
        }
#pragma unroll
        for (int i = 0; i < BPT; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float2 f = Conv<T>::to_f2(xw[i][j]);
                ss += f.x * f.x + f.y * f.y;
            }
    } else {
        for (int v = threadIdx.x; v < K / 8; v += blockDim.x) {
            const uint4 u = ld_nc_v4(xr + (size_t)v * 8);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = Conv<T>::to_f2(w[i]);
                ss += f.x * f.x + f.y * f.y;
            }
        }
    }
    ss = block_reduce(ss, false, sh);
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
    const float g = *a_global;
    if constexpr (BPT > 0) {
#pragma unroll
        for (int i = 0; i < BPT; ++i) {
            const int kb = threadIdx.x + i * blockDim.x;
            if (kb < nb) rmsnorm_nvfp4_block<T, GAMMA>(xw[i], gamma, kb, inv, g, cr, sf, row, nb);
        }
    } else {
        for (int kb = threadIdx.x; kb < nb; kb += blockDim.x) {
            const uint4 u0 = ld_nc_v4(xr + (size_t)kb * 16), u1 = ld_nc_v4(xr + (size_t)kb * 16 + 8);
            const uint32_t wv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
            rmsnorm_nvfp4_block<T, GAMMA>(wv, gamma, kb, inv, g, cr, sf, row, nb);
        }
    }
}

static __device__ unsigned int g_rn_timeout;  // a bounded wait expired in the streaming producer

// Streaming form of the producer for rows up to kRnStreamMaxK values: a
// persistent grid; each CTA walks rows blockIdx.x, + gridDim.x, ... and keeps
// kRnBufs rows in flight, each brought into shared memory by one bulk copy
// (cp.async.bulk, completion on an mbarrier, bounded wait), so the next rows
// stream in while this one is reduced and quantised.  The arithmetic is the
// per-row kernel's (rmsnorm_nvfp4_block); the padding rows of the last tile get
// zero codes and scales.
constexpr int kRnBufs = 3;
constexpr int kRnStreamMaxK = 12288;  // 768 threads, one per 16-k block

template <typename T, bool GAMMA>
__global__ void __launch_bounds__(kRnStreamMaxK / 16)
rmsnorm_nvfp4_stream_kernel(const T *__restrict__ x, const T *__restrict__ gamma, float eps,
                            const float *__restrict__ a_global, uint8_t *__restrict__ codes,
                            uint8_t *__restrict__ sf, int M, int K, int rows_padded) {
    extern __shared__ __align__(128) uint8_t rn_smem[];
    __shared__ __align__(8) uint64_t full[kRnBufs];
    __shared__ float sh[32];
    const int nb = K / 16;
    const uint32_t row_bytes = (uint32_t)K * 2;
    const int nrows = M > (int)blockIdx.x ? (M - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    if (threadIdx.x == 0) {
        for (int b = 0; b < kRnBufs; ++b) mbar_init(&full[b], 1);
        fence_mbar_init();
        for (int i = 0; i < nrows && i < kRnBufs; ++i) {
            mbar_arrive_expect_tx(&full[i], row_bytes);
            bulk_load_1d(rn_smem + (size_t)i * row_bytes, x + (size_t)(blockIdx.x + i * gridDim.x) * K, row_bytes,
                         &full[i]);
        }
    }
    __syncthreads();
    const float g = *a_global;
    for (int i = 0; i < nrows; ++i) {
        const int b = i % kRnBufs;
        const int row = blockIdx.x + i * gridDim.x;
        const bool ok = mbar_wait_bounded(&full[b], (uint32_t)((i / kRnBufs) & 1));
        if (__syncthreads_or(!ok)) {  // a copy never landed: stop every thread here
            if (threadIdx.x == 0) atomicExch(&g_rn_timeout, 1u);
            break;
        }
        // thread t owns 16-k block t of the row (blockDim = nb rounded up to a warp)
        const T *xr = reinterpret_cast<const T *>(rn_smem + (size_t)b * row_bytes);
        const int kb = threadIdx.x;
        uint32_t wv[8] = {};
        if (kb < nb) {
            const uint4 u0 = *reinterpret_cast<const uint4 *>(xr + (size_t)kb * 16);
            const uint4 u1 = *reinterpret_cast<const uint4 *>(xr + (size_t)kb * 16 + 8);
            wv[0] = u0.x, wv[1] = u0.y, wv[2] = u0.z, wv[3] = u0.w;
            wv[4] = u1.x, wv[5] = u1.y, wv[6] = u1.z, wv[7] = u1.w;
        }
        __syncthreads();  // the row is in registers: buffer b takes the row kRnBufs ahead
        if (threadIdx.x == 0 && i + kRnBufs < nrows) {
            fence_proxy_async();  // generic reads of buffer b before the copy that overwrites it
            mbar_arrive_expect_tx(&full[b], row_bytes);
            bulk_load_1d(rn_smem + (size_t)b * row_bytes, x + (size_t)(row + kRnBufs * gridDim.x) * K, row_bytes,
                         &full[b]);
        }
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float2 f = Conv<T>::to_f2(wv[j]);
            ss += f.x * f.x + f.y * f.y;
        }
        ss = block_reduce(ss, false, sh);
        const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
        if (kb < nb) rmsnorm_nvfp4_block<T, GAMMA>(wv, gamma, kb, inv, g, codes + (size_t)row * (K / 2), sf, row, nb);
    }
    // padding rows of the last 128-row tile
    for (int row = M + blockIdx.x; row < rows_padded; row += gridDim.x) {
        uint8_t *cr = codes + (size_t)row * (K / 2);
        for (int kb = threadIdx.x; kb < nb; kb += blockDim.x) {
            sf[sf_offset<true>(row, kb, nb)] = 0;
            *reinterpret_cast<uint2 *>(cr + (size_t)kb * 8) = make_uint2(0, 0);
        }
    }
}

int take_rn_wait_status() {
    unsigned int v = 0;
    W4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_rn_timeout, sizeof(v)));
    if (v) {
        const unsigned int zero = 0;
        W4_CUDA_TRY(cudaMemcpyToSymbol(g_rn_timeout, &zero, sizeof(zero)));
        set_error("a bulk copy never completed in the RMSNorm -> NVFP4 producer within the time limit");
        return W4_ERR_TIMEOUT;
    }
    return W4_OK;
}

template <typename T, bool GAMMA>
static int launch_rmsnorm_nvfp4(const T *x, const T *gamma, float eps, const float *a_global, uint8_t *codes,
                                uint8_t *sf_atoms, int M, int K, cudaStream_t st) {
    const int rows = (M + 127) / 128 * 128, nb = K / 16;
    if (K <= kRnStreamMaxK && M >= 2 * num_sms()) {
        auto kern = rmsnorm_nvfp4_stream_kernel<T, GAMMA>;
        const size_t smem = (size_t)kRnBufs * K * 2;
        {
            static std::mutex mu;
            static bool set_dev[128] = {};
            int dev = 0;
            W4_CUDA_TRY(cudaGetDevice(&dev));
            std::lock_guard<std::mutex> lk(mu);
            if (dev < 128 && !set_dev[dev]) {
                W4_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 kRnBufs * kRnStreamMaxK * 2));
                set_dev[dev] = true;
            }
        }
        const int threads = (nb + 31) / 32 * 32;
        int per_sm = 0;
        W4_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem));
        if (per_sm < 1) per_sm = 1;
        const int grid = per_sm * num_sms() < M ? per_sm * num_sms() : M;
        kern<<<grid, threads, smem, st>>>(x, gamma, eps, a_global, codes, sf_atoms, M, K, rows);
        W4_LAUNCH_CHECK();
        return W4_OK;
    }
    if (nb <= 128 * 4)
        rmsnorm_nvfp4_kernel<T, GAMMA, 4><<<rows, 128, 0, st>>>(x, gamma, eps, a_global, codes, sf_atoms, M, K);
    else if (nb <= 256 * 8)
        rmsnorm_nvfp4_kernel<T, GAMMA, 8><<<rows, 256, 0, st>>>(x, gamma, eps, a_global, codes, sf_atoms, M, K);
    else
        rmsnorm_nvfp4_kernel<T, GAMMA, 0><<<rows, 256, 0, st>>>(x, gamma, eps, a_global, codes, sf_atoms, M, K);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

int rmsnorm_nvfp4(const void *x, int x_dtype, const void *gamma, float eps, const float *a_global, uint8_t *codes,
                  uint8_t *sf_atoms, int M, int K, cudaStream_t st) {
    if (x_dtype == W4_BF16) {
        using T = __nv_bfloat16;
        if (gamma)
            return launch_rmsnorm_nvfp4<T, true>(static_cast<const T *>(x), static_cast<const T *>(gamma), eps, a_global,
                                          codes, sf_atoms, M, K, st);
        else
            return launch_rmsnorm_nvfp4<T, false>(static_cast<const T *>(x), nullptr, eps, a_global, codes, sf_atoms, M,
                                           K, st);
    } else {
        using T = __half;
        if (gamma)
            return launch_rmsnorm_nvfp4<T, true>(static_cast<const T *>(x), static_cast<const T *>(gamma), eps, a_global,
                                          codes, sf_atoms, M, K, st);
        else
            return launch_rmsnorm_nvfp4<T, false>(static_cast<const T *>(x), nullptr, eps, a_global, codes, sf_atoms, M,
                                           K, st);
    }
}

int nvfp4_quant_act(const uint16_t *a, int M, int K, const float *a_global, uint8_t *codes,
                    uint8_t *sf, cudaStream_t st) {
    const long nblk = (long)M * (K / 16);
    nvfp4_quant_act_kernel<false><<<(unsigned)((nblk + 255) / 256), 256, 0, st>>>(a, M, K, a_global, codes, sf, M);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

int nvfp4_quant_act_atoms(const uint16_t *a, int M, int K, const float *a_global, uint8_t *codes,
                          uint8_t *sf_atoms, cudaStream_t st) {
    const int rows = (M + 127) / 128 * 128;
    const long nblk = (long)rows * (K / 16);
    nvfp4_quant_act_kernel<true><<<(unsigned)((nblk + 255) / 256), 256, 0, st>>>(a, M, K, a_global, codes, sf_atoms,
                                                                                  rows);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

// ---- reference LUT kernel contract (nibble_lut_sc.cpp:198-290, oracle :319-330) ----
// Integer products summed in fp32 are exact (|acc| < 2^24), and the epilogue
// keeps the host's operation order, so the f16 result is bit-identical.
__global__ void nvfp4_lut_s8a_kernel(const int8_t *__restrict__ a, const uint8_t *__restrict__ p,
                                     const float *__restrict__ a_s, const float *__restrict__ b_s,
                                     uint16_t *__restrict__ c, int rows, int cols, int dk) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    const int r = blockIdx.y;
    if (col >= cols) return;
    const int8_t *ar = a + (size_t)r * dk;
    float acc = 0.f;
    for (int k = 0; k < dk; k += 2) {
        const uint32_t byte = p[(size_t)(k / 2) * cols + col];
        const float q0 = 2.0f * e2m1_to_f(byte & 15), q1 = 2.0f * e2m1_to_f(byte >> 4);
        acc = __fadd_rn(acc, __fmul_rn((float)ar[k], q0));
        acc = __fadd_rn(acc, __fmul_rn((float)ar[k + 1], q1));
    }
    c[(size_t)r * cols + col] = __half_as_ushort(__float2half_rn(__fmul_rn(__fmul_rn(acc, a_s[r]), b_s[col])));
}

int nvfp4_lut_s8a(const int8_t *a, const uint8_t *packed, const float *a_s, const float *b_s,
                  uint16_t *c, int rows, int cols, int dk, cudaStream_t st) {
    dim3 block(128), grid((cols + 127) / 128, rows);
    nvfp4_lut_s8a_kernel<<<grid, block, 0, st>>>(a, packed, a_s, b_s, c, rows, cols, dk);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

// ---- load-time layout transpose KN [K/2, N] -> NK [N, K/2] ----
__global__ void nvfp4_kn_to_nk_kernel(const uint8_t *__restrict__ in, int K, int N,
                                      uint8_t *__restrict__ out) {
    __shared__ uint8_t tile[32][33];
    const int kb0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;
    for (int j = ty; j < 32; j += blockDim.y) {
        const int kb = kb0 + j, n = n0 + tx;
        tile[j][tx] = (kb < K / 2 && n < N) ? in[(size_t)kb * N + n] : 0;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += blockDim.y) {
        const int n = n0 + j, kb = kb0 + tx;
        if (n < N && kb < K / 2) out[(size_t)n * (K / 2) + kb] = tile[tx][j];
    }
}

int nvfp4_kn_to_nk(const uint8_t *in, int K, int N, uint8_t *out, cudaStream_t st) {
    dim3 block(32, 8), grid((N + 31) / 32, (K / 2 + 31) / 32);
    nvfp4_kn_to_nk_kernel<<<grid, block, 0, st>>>(in, K, N, out);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

// ---------------------------------------------------------------------------
// Decode GEMM (M small) on the NK layout, bf16 warp MMA, swap-AB.
//
// A warp owns 32 output columns; lane (g = lane/4, t = lane%4) streams 16 B of
// each of the columns n0+g, n0+8+g, n0+16+g, n0+24+g per step of 128 k (lane t
// holds k 32t..32t+31 of the step, so a quad reads 64 contiguous bytes of a
// column).  MMA m-tile 0 has rows (g, g+8) = columns (n0+g, n0+8+g), m-tile 1
// columns (n0+16+g, n0+24+g).  k-step s of lane t covers k = 32t + 4s .. +3:
// slots (2t, 2t+1) <- k (+0, +1) and (2t+8, 2t+9) <- k (+2, +3), so the
// activation fragment is 8 contiguous bytes and needs no shuffling.
//
// E2M1 -> bf16 is a register lookup: two byte-permutes read the low / high
// byte of the bf16 pattern of |e2m1| from 8-entry tables held in immediates,
// a third merges the sign bytes.  The block scale (E4M3 -> bf16, exact) is then
// applied with one bf16x2 multiply; e2m1 * e4m3 needs at most 6 significant
// bits, so the weight operand is exact and only the fp32 accumulation rounds.
// The tensor scale multiplies the fp32 result.
// ---------------------------------------------------------------------------
template <int SCALE_DT>
__device__ __forceinline__ uint32_t load_scale2(const void *scale, size_t i) {
    uint32_t h;
    if constexpr (SCALE_DT == W4_E4M3) {
        const uint32_t b = __ldg(reinterpret_cast<const uint8_t *>(scale) + i);
        h = __bfloat16_as_ushort(__float2bfloat16_rn(e4m3_to_f(b)));
    } else {
        h = __ldg(reinterpret_cast<const uint16_t *>(scale) + i);
    }
    return h | (h << 16);
}

constexpr int kFp4Warps = 8;

template <int NT, int D, int SCALE_DT>
__global__ void __launch_bounds__(kFp4Warps * 32)
nvfp4_gemv_nk_kernel(const __nv_bfloat16 *__restrict__ A, const uint8_t *__restrict__ W,
                     const void *__restrict__ scale, const float *__restrict__ global_scale,
                     void *__restrict__ C, int c_dtype, int M, int N, int K, int steps_per_part,
                     int ks) {
    constexpr int NE = 2 * NT * 4;
    __shared__ float red[kFp4Warps][NE][32];
    __shared__ float part[NE * 32];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * 32;
    const int tok0 = blockIdx.z * 8 * NT;
    const int nsteps_total = K / 128;
    const int p = blockIdx.y * kFp4Warps + warp;
    const int s_begin = min(p * steps_per_part, nsteps_total);
    const int s_end = min(s_begin + steps_per_part, nsteps_total);
    const int nsteps = s_end - s_begin;
    const size_t kb2 = (size_t)K / 2;

    float acc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[a][b][i] = 0.f;

    // column c in 0..3 of this lane: n0 + g + 8c
    const uint8_t *wp = W + (size_t)(n0 + g) * kb2 + (size_t)s_begin * 64 + 16 * t;
    uint4 wbuf[D][4];
#pragma unroll
    for (int d = 0; d < D; ++d)
        if (d < nsteps)
#pragma unroll
            for (int c = 0; c < 4; ++c) wbuf[d][c] = ld_stream_v4(wp + (size_t)(8 * c) * kb2 + d * 64);

    for (int i0 = 0; i0 < nsteps; i0 += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
            const int step = i0 + d;
            if (step < nsteps) {
                uint4 wv[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) wv[c] = wbuf[d][c];
                if (step + D < nsteps)
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        wbuf[d][c] = ld_stream_v4(wp + (size_t)(8 * c) * kb2 + (size_t)(step + D) * 64);
                const int kstep = (s_begin + step) * 128;  // first k of this step
                // block scales: blocks (kstep/16 + 2t + {0,1}) for the 4 columns
                uint32_t sc[4][2];
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        sc[c][h] = load_scale2<SCALE_DT>(scale, (size_t)(kstep / 16 + 2 * t + h) * N + n0 + g + 8 * c);
                // activations: 32 bf16 per token starting at kstep + 32t
                uint4 xa[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int tok = tok0 + nt * 8 + g;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        xa[nt][q] = (tok < M) ? ld_nc_v4(A + (size_t)tok * K + kstep + 32 * t + 8 * q)
                                              : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int s = 0; s < 8; ++s) {
                    const int q = s >> 1, half = s & 1, h = s >> 2;
                    uint32_t a01[4], a23[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t word = (q == 0) ? wv[c].x : (q == 1) ? wv[c].y : (q == 2) ? wv[c].z : wv[c].w;
                        uint32_t r01, r23;
                        e2m1x4_to_bf16(half ? (word >> 16) : word, r01, r23);
                        a01[c] = bf16x2_mul(r01, sc[c][h]);
                        a23[c] = bf16x2_mul(r23, sc[c][h]);
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const uint4 xv = xa[nt][q];
                        const uint32_t b0 = half ? xv.z : xv.x, b1 = half ? xv.w : xv.y;
                        mma_16816<__nv_bfloat16>(acc[0][nt], a01[0], a01[1], a23[0], a23[1], b0, b1);
                        mma_16816<__nv_bfloat16>(acc[1][nt], a01[2], a01[3], a23[2], a23[3], b0, b1);
                    }
                }
            }
        }
    }

    // ---- reduce: warps -> CTA -> cluster leader (distributed shared memory) ----
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[warp][(mt * NT + nt) * 4 + i][lane] = acc[mt][nt][i];
    __syncthreads();
    for (int idx = threadIdx.x; idx < NE * 32; idx += blockDim.x) {
        const int e = idx >> 5, l = idx & 31;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kFp4Warps; ++w) v += red[w][e][l];
        part[idx] = v;
    }
    bool leader = true;
    if (ks > 1) {
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        leader = cluster.block_rank() == 0;
        if (leader) {
            for (int idx = threadIdx.x; idx < NE * 32; idx += blockDim.x) {
                float v = part[idx];
                for (int r = 1; r < ks; ++r) v += cluster.map_shared_rank(part, r)[idx];
                red[0][0][idx] = v;
            }
        }
        cluster.sync();
    } else {
        __syncthreads();
    }
    if (!leader) return;
    const float gsc = global_scale ? *global_scale : 1.0f;
    const float *src = (ks > 1) ? &red[0][0][0] : part;
    for (int idx = threadIdx.x; idx < NE * 32; idx += blockDim.x) {
        const int e = idx >> 5, l = idx & 31;
        const int mt = e / (NT * 4), nt = (e / 4) % NT, i = e & 3;
        const int col = n0 + 16 * mt + 8 * (i >> 1) + (l >> 2);
        const int tok = tok0 + nt * 8 + 2 * (l & 3) + (i & 1);
        if (tok < M && col < N) {
            const float v = src[idx] * gsc;
            const size_t o = (size_t)tok * N + col;
            if (c_dtype == W4_F32) reinterpret_cast<float *>(C)[o] = v;
            else if (c_dtype == W4_BF16) reinterpret_cast<__nv_bfloat16 *>(C)[o] = __float2bfloat16_rn(v);
            else reinterpret_cast<__half *>(C)[o] = __float2half_rn(v);
        }
    }
}

template <int NT, int SCALE_DT>
static int launch_nvfp4_gemv_t(const uint16_t *a, const uint8_t *w, const void *scale,
                               const float *global_scale, void *c, int c_dtype, int M, int N,
                               int K, cudaStream_t st) {
    constexpr int D = 2;
    const int nsm = num_sms();
    const int ncol = N / 32;
    const int mblocks = (M + 8 * NT - 1) / (8 * NT);
    const int nsteps = K / 128;
    int ks = 1;
    while (ks < 8 && ncol * mblocks * ks < 2 * nsm && nsteps / (kFp4Warps * ks * 2) >= 1) ks *= 2;
    const int spp = (nsteps + kFp4Warps * ks - 1) / (kFp4Warps * ks);

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ncol, ks, mblocks);
    cfg.blockDim = dim3(kFp4Warps * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = ks;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ks > 1 ? 1 : 0;
    W4_CUDA_TRY(cudaLaunchKernelEx(&cfg, nvfp4_gemv_nk_kernel<NT, D, SCALE_DT>,
                                   reinterpret_cast<const __nv_bfloat16 *>(a), w, scale,
                                   global_scale, c, c_dtype, M, N, K, spp, ks));
    return W4_OK;
}

int nvfp4_gemv(const uint16_t *a, const uint8_t *w, int layout, const void *scale,
               int scale_dtype, const float *global_scale, void *c, int c_dtype, int M, int N,
               int K, void *sync, void *ws, size_t ws_bytes, cudaStream_t st) {
    (void)layout;  // NK only; validated by the caller
    // the TMA-ring kernel (nvfp4_decode.cu) first; the register-streamed one below covers
    // pointers it does not take
    const int rc = nvfp4_gemv_decode(a, w, scale, scale_dtype, global_scale, c, c_dtype, M, N, K, sync, ws,
                                     ws_bytes, nullptr, st);
    if (rc >= 0) return rc;
    note_decode_fallback();
    if (scale_dtype == W4_E4M3) {
        if (M <= 8) return launch_nvfp4_gemv_t<1, W4_E4M3>(a, w, scale, global_scale, c, c_dtype, M, N, K, st);
        if (M <= 16) return launch_nvfp4_gemv_t<2, W4_E4M3>(a, w, scale, global_scale, c, c_dtype, M, N, K, st);
        return launch_nvfp4_gemv_t<4, W4_E4M3>(a, w, scale, global_scale, c, c_dtype, M, N, K, st);
    }
    if (M <= 8) return launch_nvfp4_gemv_t<1, W4_BF16>(a, w, scale, global_scale, c, c_dtype, M, N, K, st);
    if (M <= 16) return launch_nvfp4_gemv_t<2, W4_BF16>(a, w, scale, global_scale, c, c_dtype, M, N, K, st);
    return launch_nvfp4_gemv_t<4, W4_BF16>(a, w, scale, global_scale, c, c_dtype, M, N, K, st);
}

}  // namespace w4
