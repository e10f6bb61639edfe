// nvfp4_tma.cu -- NVFP4 W4A16 decode GEMM with TMA-streamed operands (sm_100a).
//
// Contract: w4_nvfp4_gemm with act_mode W4A16 on the K-contiguous layout,
//   C[m,n] = (sum_k A[m,k] * (e2m1(w[n,k]) * s[k/16,n])) * global
// (the external operator nvfp4_gemm_w4a16[_f8scale], kernels/nvfp4/bench_nvfp4_m1.py:67,88;
// the reference LUT kernel's host loop kernels/nvfp4/nibble_lut_sc.cpp:319-330
// without the block scales).
//
// Same organisation as the GPTQ decode kernel (gptq_tma.cu): a CTA owns 32
// output columns; W consumer warps split K in stages of 256 k; one producer
// warp streams, per stage, the weight tile (32 rows x 128 bytes of [N, K/2],
// 128-byte swizzled), the 16 x 32 block scales and the activation rows (3-D
// swizzled box) into the consumer's ring, completing on one mbarrier.
//
// Consumer math (bf16 warp MMA, swap-AB): lane (g = lane/4, t = lane%4) owns
// the weight columns n0 + 4g + c (c = 0..3: m-tile 0 rows g / g+8 are columns
// 4g / 4g+1, m-tile 1 columns 4g+2 / 4g+3) and k 32t..32t+31 of each 128-k
// step, so its four block scales of a 16-k block are one 32-bit word.  k-step s
// covers k = 32t + 4s .. +3 (slots 2t, 2t+1 <- +0, +1 and 2t+8, 2t+9 <- +2, +3),
// so the activation fragment is 8 contiguous bytes.  E2M1 -> bf16 is a register
// lookup (nvfp4_util.cuh); E4M3 -> bf16 goes through the hardware fp8 -> f16
// conversion (exact); e2m1 * e4m3 has at most 6 significant bits, so the MMA
// operand is exact and only the fp32 accumulation rounds.  The tensor scale
// multiplies the fp32 sum.  Every wait is bounded (tma_util.cuh); no copy uses
// multicast.
#include <cuda_fp8.h>

#include <mutex>

#include "nvfp4_util.cuh"
#include "tma_util.cuh"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

static __device__ unsigned int g_fp4_timeout;  // a bounded wait expired (sticky until read)

namespace fp4t {

constexpr int S = 3;            // ring depth per consumer warp
constexpr int KS = 256;         // k per stage (two 128-k steps)
constexpr int kMaxWarps = 8;    // consumer warps per CTA (one more warp produces)
// Register cap: 128 lets 4 CTAs of 4 warps share an SM; two token tiles (NT = 2)
// need more to keep both activation fragments and accumulators in registers.
template <int NT> constexpr int max_regs() { return NT == 1 ? 128 : 192; }

// Byte offsets inside one consumer warp's ring (from a 1024-aligned base).
struct Lay {
    uint32_t act_stage, sc_stage, act, sc, bars, red, total;
    static constexpr uint32_t W_STAGE = 32 * 128;  // 32 columns x 256 k of nibbles
    __host__ __device__ Lay(int act_rows, int scale_bytes, int red_bytes) {
        act_stage = (act_rows * KS * 2 + 1023) & ~1023;
        sc_stage = (16 * 32 * scale_bytes + 127) & ~127;
        act = S * W_STAGE;
        sc = act + S * act_stage;
        bars = sc + S * sc_stage;
        red = (bars + 2 * S * 8 + 127) & ~127u;
        total = (red + red_bytes + 1023) & ~1023u;
    }
};

__device__ __forceinline__ bool wait_fp4(uint64_t *bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicExch(&g_fp4_timeout, 1u);
    return false;
}

__device__ __forceinline__ uint32_t bf16_pair(float x) {
    const uint32_t u = __bfloat16_as_ushort(__float2bfloat16_rn(x));
    return u | (u << 16);
}

// Four block scales (columns 4g + c, c = 0..3) -> bf16 pairs broadcast to both halves.
template <int SDT> __device__ __forceinline__ void load_scales4(const uint8_t *p, uint32_t (&sc)[4]) {
    if constexpr (SDT == W4_E4M3) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
        const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xFFFFu), __NV_E4M3);
        const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3);
        sc[0] = bf16_pair(__half2float(__ushort_as_half(lo.x)));
        sc[1] = bf16_pair(__half2float(__ushort_as_half(lo.y)));
        sc[2] = bf16_pair(__half2float(__ushort_as_half(hi.x)));
        sc[3] = bf16_pair(__half2float(__ushort_as_half(hi.y)));
    } else {
        const uint2 w = *reinterpret_cast<const uint2 *>(p);
        sc[0] = __byte_perm(w.x, 0, 0x1010);
        sc[1] = __byte_perm(w.x, 0, 0x3232);
        sc[2] = __byte_perm(w.y, 0, 0x1010);
        sc[3] = __byte_perm(w.y, 0, 0x3232);
    }
}

template <int NT, int SDT>
__global__ void __maxnreg__(max_regs<NT>())
nvfp4_gemv_tma_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap sc_map,
                      const __grid_constant__ CUtensorMap act_map, const float *__restrict__ global_scale,
                      void *__restrict__ C, int c_dtype, int M, int N, int stages_all, int act_rows, int pre) {
    constexpr int NE = 2 * NT * 4;
    constexpr int SB = SDT == W4_E4M3 ? 1 : 2;  // bytes per block scale
    extern __shared__ uint8_t smem_dyn[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int W = (blockDim.x >> 5) - 1;
    const Lay L(act_rows, SB, NE * 32 * 4);
    const int n0 = blockIdx.y * 32;
    const int tok0 = blockIdx.x * 8 * NT;
    // Split K across the CTAs of a cluster (grid z): this CTA owns stages
    // [zb, zb + stages_total) of the stages_all stages of K.
    const int zb = (int)(blockIdx.z * (unsigned)stages_all / gridDim.z);
    const int stages_total = (int)((blockIdx.z + 1) * (unsigned)stages_all / gridDim.z) - zb;

    if (warp == W && lane == 0) {
        for (int w = 0; w < W; ++w) {
            uint64_t *bars = reinterpret_cast<uint64_t *>(base + (size_t)w * L.total + L.bars);
            for (int i = 0; i < 2 * S; ++i) mbar_init(&bars[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == W) {  // ---------------- producer ----------------
        if (lane == 0) {
            const uint32_t tx = Lay::W_STAGE + act_rows * KS * 2 + 16 * 32 * SB;
            bool ok = true;
            const int most = (stages_total + W - 1) / W;
            // pre: codes and block scales of the first ring fill are requested before
            // the previous kernel on the stream has completed (static weights).
            const int pf = pre ? (most < S ? most : S) : 0;
            for (int it = 0; it < pf; ++it)
                for (int w = 0; w < W; ++w) {
                    const int sb = w * stages_total / W, se = (w + 1) * stages_total / W;
                    if (sb + it >= se) continue;
                    uint8_t *r = base + (size_t)w * L.total;
                    uint64_t *full = reinterpret_cast<uint64_t *>(r + L.bars) + it;
                    mbar_arrive_expect_tx(full, tx);
                    tma_load_2d(r + it * Lay::W_STAGE, &w_map, (zb + sb + it) * (KS / 2), n0, full);
                    tma_load_2d(r + L.sc + it * L.sc_stage, &sc_map, n0, (zb + sb + it) * (KS / 16), full);
                }
            grid_dep_wait();  // activations are the previous kernel's output
            for (int it = 0; it < most && ok; ++it) {
                const int s = it % S;
                for (int w = 0; w < W && ok; ++w) {
                    const int sb = w * stages_total / W, se = (w + 1) * stages_total / W;
                    if (sb + it >= se) continue;
                    uint8_t *r = base + (size_t)w * L.total;
                    uint64_t *full = reinterpret_cast<uint64_t *>(r + L.bars) + s;
                    const int st = zb + sb + it;
                    if (it >= pf) {
                        if (it >= S && !wait_fp4(full + S, (uint32_t)(((it / S) - 1) & 1))) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(full, tx);
                        tma_load_2d(r + s * Lay::W_STAGE, &w_map, st * (KS / 2), n0, full);
                        tma_load_2d(r + L.sc + s * L.sc_stage, &sc_map, n0, st * (KS / 16), full);
                    }
                    tma_load_3d(r + L.act + s * L.act_stage, &act_map, 0, tok0, st * (KS / 64), full);
                }
            }
        }
        __syncwarp();
        grid_dep_launch();  // every copy is issued: the next decode GEMM may be scheduled
        if (gridDim.z > 1) {  // meet the consumers at the cluster reduction's two barriers
            cluster_sync_all();
            cluster_sync_all();
        }
        return;
    }
    grid_dep_wait();  // nothing below touches global memory before the previous kernel completed

    // ---------------- consumers ----------------
    uint8_t *ring = base + (size_t)warp * L.total;
    uint64_t *fullb = reinterpret_cast<uint64_t *>(ring + L.bars);
    float *red = reinterpret_cast<float *>(ring + L.red);
    const int g = lane >> 2, t = lane & 3;
    const int sbeg = warp * stages_total / W;
    const int nstages = (warp + 1) * stages_total / W - sbeg;
    // weights: row 4g + c, 16-byte chunk 4h + t of step h, swizzled by row % 8
    uint32_t woff[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int r = 4 * g + c;
            woff[h][c] = r * 128 + (((4 * h + t) ^ (r & 7)) << 4);
        }
    // activations: k = 128h + 32t + 8q of the stage -> line (2h + t/2) of the token row
    uint32_t aoff[2][4][NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int row = (nt * 8 + g) < act_rows ? nt * 8 + g : 0;  // rows past the box: outputs discarded
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int line = (2 * h + (t >> 1)) * act_rows + row;
                aoff[h][q][nt] = line * 128 + (((4 * (t & 1) + q) ^ (line & 7)) << 4);
            }
    }

    float acc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[a][b][i] = 0.f;

    uint32_t parity = 0;
    bool ok = true;
    for (int it0 = 0; it0 < nstages && ok; it0 += S, parity ^= 1u) {
#pragma unroll
        for (int s = 0; s < S; ++s) {
            if (it0 + s < nstages && ok) {
                if (!__all_sync(0xffffffffu, wait_fp4(&fullb[s], parity))) {
                    ok = false;
                } else {
                    const uint8_t *ws = ring + s * Lay::W_STAGE;
                    const uint8_t *as = ring + L.act + s * L.act_stage;
                    const uint8_t *ss = ring + L.sc + s * L.sc_stage;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint4 wv[4];
#pragma unroll
                        for (int c = 0; c < 4; ++c) wv[c] = *reinterpret_cast<const uint4 *>(ws + woff[h][c]);
                        uint32_t sc[2][4];
#pragma unroll
                        for (int hb = 0; hb < 2; ++hb)
                            load_scales4<SDT>(ss + ((8 * h + 2 * t + hb) * 32 + 4 * g) * SB, sc[hb]);
                        uint4 xa[NT][4];
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int q = 0; q < 4; ++q) xa[nt][q] = *reinterpret_cast<const uint4 *>(as + aoff[h][q][nt]);
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const int q = k >> 1, half = k & 1, hb = k >> 2;
                            uint32_t a01[4], a23[4];
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                const uint32_t word = q == 0 ? wv[c].x : q == 1 ? wv[c].y : q == 2 ? wv[c].z : wv[c].w;
                                uint32_t r01, r23;
                                e2m1x4_to_bf16(half ? (word >> 16) : word, r01, r23);
                                a01[c] = bf16x2_mul(r01, sc[hb][c]);
                                a23[c] = bf16x2_mul(r23, sc[hb][c]);
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
                    __syncwarp();
                    if (lane == 0)
                        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&fullb[S + s])) : "memory");
                }
            }
        }
    }

    // The next decode GEMM may be scheduled once every thread of every CTA is here
    // (late, so its CTAs take the slots this grid frees, evenly).
    grid_dep_launch();
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[((mt * NT + nt) * 4 + i) * 32 + lane] = acc[mt][nt][i];
    asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
    const float gsc = global_scale ? *global_scale : 1.0f;
    if (gridDim.z == 1) {
        for (int idx = threadIdx.x; idx < NE * 32; idx += W * 32) {
            float v = 0.f;
            for (int w = 0; w < W; ++w) v += reinterpret_cast<const float *>(base + (size_t)w * L.total + L.red)[idx];
            const int e = idx >> 5, l = idx & 31;
            const int mt = e / (NT * 4), nt = (e / 4) % NT, i = e & 3;
            const int col = n0 + 4 * (l >> 2) + 2 * mt + (i >> 1);
            const int tok = tok0 + nt * 8 + 2 * (l & 3) + (i & 1);
            if (tok < M) store_out(C, c_dtype, (size_t)tok * N + col, v * gsc);
        }
    } else {
        // K split over the cluster: partial tiles stay in each CTA's shared memory;
        // CTA r sums elements r, r + ks, ... over the cluster in rank order.
        float *fin = reinterpret_cast<float *>(base + (size_t)W * L.total);
        for (int idx = threadIdx.x; idx < NE * 32; idx += W * 32) {
            float v = 0.f;
            for (int w = 0; w < W; ++w) v += reinterpret_cast<const float *>(base + (size_t)w * L.total + L.red)[idx];
            fin[idx] = v;
        }
        cluster_sync_all();
        const int ks = (int)gridDim.z, cr = (int)cluster_rank();
        for (int idx = cr + ks * (int)threadIdx.x; idx < NE * 32; idx += ks * W * 32) {
            float v = 0.f;
            for (int c = 0; c < ks; ++c) v += ld_cluster_f32(fin + idx, (uint32_t)c);
            const int e = idx >> 5, l = idx & 31;
            const int mt = e / (NT * 4), nt = (e / 4) % NT, i = e & 3;
            const int col = n0 + 4 * (l >> 2) + 2 * mt + (i >> 1);
            const int tok = tok0 + nt * 8 + 2 * (l & 3) + (i & 1);
            if (tok < M) store_out(C, c_dtype, (size_t)tok * N + col, v * gsc);
        }
        cluster_sync_all();  // no CTA leaves while another still reads its tile
    }
}

template <int NT, int SDT>
static int launch(const uint16_t *a, const uint8_t *w, const void *scale, const float *global_scale, void *c,
                  int c_dtype, int M, int N, int K, cudaStream_t st) {
    constexpr int NE = 2 * NT * 4;
    constexpr int SB = SDT == W4_E4M3 ? 1 : 2;
    if (K % KS) return -1;
    const int nsm = num_sms();
    const int nchunk = N / 32;
    const int mblocks = (M + 8 * NT - 1) / (8 * NT);
    const int stages_total = K / KS;
    const int act_rows = M < 8 * NT ? M : 8 * NT;
    const Lay lay(act_rows, SB, NE * 32 * 4);
    const long ctas = (long)nchunk * mblocks;
    // Fewer column tiles than two per SM: split K over a cluster of ks CTAs per
    // tile (reduced through distributed shared memory).
    int ks = 1;
    if (ctas < 2L * nsm) {
        ks = (int)((2L * nsm + ctas - 1) / ctas);
        if (ks > 4) ks = 4;
        if (ks > stages_total) ks = stages_total;
    }
    const size_t fin_bytes = ks > 1 ? (size_t)NE * 32 * 4 : 0;
    const long ctas_per_sm = (ctas * ks + nsm - 1) / nsm;
    long fit = ((224L * 1024) / ctas_per_sm - 1024 - (long)fin_bytes) / (long)lay.total;
    const long fit_regs = 65536L / (ctas_per_sm * 32L * max_regs<NT>()) - 1;  // the register file too
    if (fit_regs < fit) fit = fit_regs;
    int W = (int)(fit < 1 ? 1 : (fit > kMaxWarps ? kMaxWarps : fit));
    if (W > stages_total / ks) W = stages_total / ks;  // every warp of every CTA gets a stage
    CUtensorMap w_map, sc_map, act_map;
    if (!make_map_2d(&w_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)K / 2, N, (uint64_t)K / 2, KS / 2, 32,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&sc_map, SB == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, scale, N,
                     K / 16, (uint64_t)N * SB, 32, 16, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_act_map(&act_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a, M, K, act_rows, KS / 64))
        return -1;
    auto kern = nvfp4_gemv_tma_kernel<NT, SDT>;
    {
        static std::mutex mu;
        static bool set_dev[128] = {};
        int dev = 0;
        W4_CUDA_TRY(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lk(mu);
        if (dev < 128 && !set_dev[dev]) {
            W4_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
            W4_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
            set_dev[dev] = true;
        }
    }
    const size_t smem = 1024 + (size_t)W * lay.total + fin_bytes;
    if (smem > 220 * 1024) return -1;
    dim3 grid(mblocks, nchunk, ks), block(32 * (W + 1));
    const int pre = launch_overlap() == W4_OVERLAP_STATIC_WEIGHTS;
    W4_CUDA_TRY(launch_decode(kern, grid, block, smem, st, (unsigned)ks, w_map, sc_map, act_map, global_scale, c, c_dtype, M, N,
                              stages_total, act_rows, pre));
    return W4_OK;
}

}  // namespace fp4t

// W4_OK / a W4 error, or -1 when the shape or tensor maps are not handled here
// (the caller then runs the register-streamed kernel).
int nvfp4_gemv_tma(const uint16_t *a, const uint8_t *w, const void *scale, int scale_dtype,
                   const float *global_scale, void *c, int c_dtype, int M, int N, int K, cudaStream_t st) {
    if (scale_dtype == W4_E4M3)
        return M <= 8 ? fp4t::launch<1, W4_E4M3>(a, w, scale, global_scale, c, c_dtype, M, N, K, st)
                      : fp4t::launch<2, W4_E4M3>(a, w, scale, global_scale, c, c_dtype, M, N, K, st);
    return M <= 8 ? fp4t::launch<1, W4_BF16>(a, w, scale, global_scale, c, c_dtype, M, N, K, st)
                  : fp4t::launch<2, W4_BF16>(a, w, scale, global_scale, c, c_dtype, M, N, K, st);
}

int take_fp4_wait_status() {
    unsigned int v = 0;
    W4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_fp4_timeout, sizeof(v)));
    if (v) {
        const unsigned int zero = 0;
        W4_CUDA_TRY(cudaMemcpyToSymbol(g_fp4_timeout, &zero, sizeof(zero)));
        set_error("a device-side wait expired in the NVFP4 decode GEMM");
        return W4_ERR_TIMEOUT;
    }
    return W4_OK;
}

}  // namespace w4
