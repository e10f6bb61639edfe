// gptq.cu -- GPTQ int4 kernels for sm_100a.
//
// Checkpoint layout (kernels/nvfp4/gptq_s4_dump.py:106-114 of the reference):
//   qweight i32 [K/8, N]   eight 4-bit codes per word, LSB-first along K
//   qzeros  i32 [K/gs, N/8] eight codes per word, LSB-first along N (or absent)
//   scales  f16 [K/gs, N]
// The kernels read this layout as stored; nothing is repacked for the GEMM
// except the optional act_order row permutation.
#include <cooperative_groups.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "w4_common.cuh"
#include "w4_internal.h"

namespace cg = cooperative_groups;

namespace w4 {

// ---------------------------------------------------------------------------
// Dequantisation (bit-exact): one thread per qweight word -> 8 fp32 outputs.
// ---------------------------------------------------------------------------
__global__ void gptq_dequant_kernel(const int32_t *__restrict__ qweight,
                                    const int32_t *__restrict__ qzeros,
                                    const uint16_t *__restrict__ scales,
                                    const int32_t *__restrict__ g_idx, int K, int N, int gs,
                                    int zero_offset, float *__restrict__ w) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int kw = blockIdx.y;
    if (n >= N) return;
    const uint32_t word = (uint32_t)qweight[(size_t)kw * N + n];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const int k = kw * 8 + s;
        const int g = g_idx ? g_idx[k] : k / gs;
        int z = 8;
        if (qzeros) z = (int)(((uint32_t)qzeros[(size_t)g * (N / 8) + (n >> 3)] >> (4 * (n & 7))) & 15u) + zero_offset;
        const int d = (int)((word >> (4 * s)) & 15u) - z;
        w[(size_t)k * N + n] = __fmul_rn((float)d, f16_bits_to_f(scales[(size_t)g * N + n]));
    }
}

int gptq_dequant(const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                 const int32_t *g_idx, int K, int N, int gs, int zero_offset, float *w,
                 cudaStream_t st) {
    dim3 block(256), grid((N + 255) / 256, K / 8);
    gptq_dequant_kernel<<<grid, block, 0, st>>>(qweight, qzeros, scales, g_idx, K, N, gs,
                                                zero_offset, w);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

// ---------------------------------------------------------------------------
// act_order repack.  perm = stable argsort(g_idx) by counting sort (one block,
// one thread per group scanning K in order), then row gather of the codes.
// ---------------------------------------------------------------------------
__global__ void act_order_perm_kernel(const int32_t *__restrict__ g_idx, int K, int gs,
                                      int32_t *__restrict__ perm) {
    __shared__ int bad;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    const int ngrp = K / gs;
    for (int g = threadIdx.x; g < ngrp; g += blockDim.x) {
        int pos = g * gs, cnt = 0;
        for (int k = 0; k < K; ++k) {
            if (g_idx[k] == g) {
                if (cnt < gs) perm[pos + cnt] = k;
                ++cnt;
            }
        }
        if (cnt != gs) atomicExch(&bad, 1);
    }
    __syncthreads();
    // A valid permutation never starts with -1: it marks an invalid g_idx.
    if (threadIdx.x == 0 && bad) perm[0] = -1;
}

__global__ void permute_rows_kernel(const int32_t *__restrict__ qweight,
                                    const int32_t *__restrict__ perm, int N,
                                    int32_t *__restrict__ out) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int kw = blockIdx.y;
    if (n >= N) return;
    uint32_t word = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const int src = perm[kw * 8 + s];
        const uint32_t v = ((uint32_t)qweight[(size_t)(src >> 3) * N + n] >> (4 * (src & 7))) & 15u;
        word |= v << (4 * s);
    }
    out[(size_t)kw * N + n] = (int32_t)word;
}

int gptq_repack_act_order(const int32_t *qweight, const int32_t *g_idx, int K, int N, int gs,
                          int32_t *qweight_out, int32_t *perm_out, cudaStream_t st) {
    act_order_perm_kernel<<<1, 256, 0, st>>>(g_idx, K, gs, perm_out);
    W4_LAUNCH_CHECK();
    // Load-time call: read the validity marker back synchronously.
    int32_t first = 0;
    W4_CUDA_TRY(cudaMemcpyAsync(&first, perm_out, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    W4_CUDA_TRY(cudaStreamSynchronize(st));
    W4_REQUIRE(first >= 0, W4_ERR_UNSUPPORTED,
               "act_order: every group must hold exactly group_size=%d rows", gs);
    dim3 block(256), grid((N + 255) / 256, K / 8);
    permute_rows_kernel<<<grid, block, 0, st>>>(qweight, perm_out, N, qweight_out);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

// A_perm[m, k] = A[m, perm[k]] (16-bit elements)
__global__ void gather_cols_kernel(const uint16_t *__restrict__ a, const int32_t *__restrict__ perm,
                                   int K, uint16_t *__restrict__ out) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    if (k >= K) return;
    out[(size_t)m * K + k] = a[(size_t)m * K + perm[k]];
}

int gather_cols(const uint16_t *a, const int32_t *perm, int M, int K, uint16_t *out,
                cudaStream_t st) {
    dim3 block(256), grid((K + 255) / 256, M);
    gather_cols_kernel<<<grid, block, 0, st>>>(a, perm, K, out);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

// ---------------------------------------------------------------------------
// Decode GEMM (M small): warp-level, HBM-bound.
//
// A warp owns 32 output columns and a run of qweight words (4 words = 32 k per
// step).  Lane (g = lane/4, t = lane%4) loads 16 B = 4 adjacent columns of word
// row (kbase + t): for each t the 8 lanes of that t read one contiguous 128-byte
// line.  The 32 codes in the lane's registers become the A operand of m16n8k16
// MMAs with the WEIGHT COLUMNS as MMA rows (swap-AB) and the tokens as MMA
// columns:
//   m-tile mt: MMA row g   <- column 4g + 2mt,  MMA row g+8 <- column 4g + 2mt + 1
//   k-step s : MMA k-slots (2t, 2t+1) <- codes (2s, 2s+4) of word kbase+t,
//              k-slots (2t+8, 2t+9) <- codes (2s+1, 2s+5)
// Any consistent relabelling of k is legal for a dot product; this one lets a
// single lop3 turn code pair (j, j+4) of a word into two 16-bit floats
// (magic + q) and the activations follow with two byte-permutes per pair.
// (q - zero) is formed exactly in bf16/f16, products are exact, fp32
// accumulation runs per group and is scaled by the fp16 group scale when the
// group ends -- the s32-partial-then-scale structure of the reference kernel
// (kernels/esimd_dpas/dpas_s4_gptq_sc.cpp:178-218) with real activations.
// ---------------------------------------------------------------------------
template <typename T> struct Deq;
template <> struct Deq<__nv_bfloat16> {
    // bf16 128.0 with q in mantissa bits 0-3 is 128 + q; (128 + z) is 0x4300 + z
    static constexpr uint32_t kMagic = 0x43004300u, kMagicHalf = 0x4300u;
    static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
        __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162 *>(&a),
                                   *reinterpret_cast<__nv_bfloat162 *>(&b));
        return *reinterpret_cast<uint32_t *>(&r);
    }
};
template <> struct Deq<__half> {
    // f16 1024.0 with q in mantissa bits 0-3 is 1024 + q; (1024 + z) is 0x6400 + z
    static constexpr uint32_t kMagic = 0x64006400u, kMagicHalf = 0x6400u;
    static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
        __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
        return *reinterpret_cast<uint32_t *>(&r);
    }
};

// Geometry: a CTA owns 32 output columns; its W warps (blockDim = 32 W, W <= 16)
// split K into W contiguous runs of whole virtual groups and meet in shared
// memory at the end.  Token blocks of 8*NT run as grid.x (fastest), so the
// token blocks of a column chunk re-read its weights from L2.
//
// Streaming: HBM on this part needs ~120 KB of reads in flight per SM (loaded
// latency ~3 us).  Each warp issues a batch of kBatch independent 16-byte
// weight loads (kBatch steps of 32 k) and then consumes the whole batch, so no
// outstanding load waits behind a younger one; W is chosen on the host so the
// whole grid is resident at once (one wave).
template <int NT> struct GemvCfg;
template <> struct GemvCfg<1> { static constexpr int kBatch = 16, kMaxRegs = 128; };
template <> struct GemvCfg<2> { static constexpr int kBatch = 8, kMaxRegs = 128; };
constexpr int kGemvMaxWarps = 16;

template <typename T, int NT, int GSTEPS>
__global__ void __launch_bounds__(kGemvMaxWarps * 32)
gptq_gemv_kernel(const T *__restrict__ A, const int32_t *__restrict__ qweight,
                 const int32_t *__restrict__ qzeros, const uint16_t *__restrict__ scales,
                 void *__restrict__ C, int c_dtype, int M, int N, int K, int zero_offset,
                 int vpg, int vgroups_per_warp) {
    constexpr int kBatch = GemvCfg<NT>::kBatch;
    static_assert(kBatch % GSTEPS == 0, "a batch holds whole virtual groups");
    constexpr int VPB = kBatch / GSTEPS;  // virtual groups per batch
    constexpr int NE = 2 * NT * 4;
    extern __shared__ float red[];  // [W][NE][32]

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int n_base = blockIdx.y * 32 + 4 * g;
    const int tok0 = blockIdx.x * 8 * NT;
    const int nvg = K / (32 * GSTEPS);
    const int vg_begin = min(warp * vgroups_per_warp, nvg);
    const int vg_end = min(vg_begin + vgroups_per_warp, nvg);
    const int nsteps = (vg_end - vg_begin) * GSTEPS;
    const int w0 = vg_begin * GSTEPS * 4;  // first qweight word row of this warp
    const bool has_z = qzeros != nullptr;
    const int zshift = 4 * (n_base & 7);

    const int step_stride = 4 * N;  // int32 elements per step (K/8 * N < 2^31 is validated)
    int woff = (w0 + t) * N + n_base;
    const T *ap[NT];
    bool av[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int tok = tok0 + nt * 8 + g;
        av[nt] = tok < M;
        ap[nt] = A + (size_t)(av[nt] ? tok : 0) * K + (size_t)(w0 + t) * 8;
    }

    float facc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) facc[a][b][i] = 0.f;

    for (int b0 = 0; b0 < nsteps; b0 += kBatch) {
        // ---- issue the whole batch: weights, then the group constants ----
        uint4 wv[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            wv[u] = make_uint4(0, 0, 0, 0);
            if (b0 + u < nsteps) wv[u] = ld_stream_v4(qweight + woff + u * step_stride);
        }
        uint32_t zw[VPB];
        uint2 sw[VPB];
#pragma unroll
        for (int v = 0; v < VPB; ++v) {
            zw[v] = 0;
            sw[v] = make_uint2(0, 0);
            if (b0 + v * GSTEPS < nsteps) {
                const int grp = (vg_begin + b0 / GSTEPS + v) / vpg;
                if (has_z) zw[v] = (uint32_t)__ldg(qzeros + grp * (N / 8) + (n_base >> 3));
                sw[v] = __ldg(reinterpret_cast<const uint2 *>(scales + grp * N + n_base));
            }
        }
        woff += kBatch * step_stride;
        // ---- consume it ----
#pragma unroll
        for (int v = 0; v < VPB; ++v) {
            if (b0 + v * GSTEPS < nsteps) {
                uint32_t zc[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t z = has_z ? ((zw[v] >> (zshift + 4 * c)) & 15u) + (uint32_t)zero_offset : 8u;
                    zc[c] = (Deq<T>::kMagicHalf + z) * 0x00010001u;
                }
                float gacc[2][NT][4];
#pragma unroll
                for (int a = 0; a < 2; ++a)
#pragma unroll
                    for (int bb = 0; bb < NT; ++bb)
#pragma unroll
                        for (int i = 0; i < 4; ++i) gacc[a][bb][i] = 0.f;
#pragma unroll
                for (int s = 0; s < GSTEPS; ++s) {
                    const int u = v * GSTEPS + s;
                    const int step = b0 + u;
                    uint32_t bf[NT][2][2];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        uint4 x = make_uint4(0, 0, 0, 0);
                        if (av[nt]) x = __ldg(reinterpret_cast<const uint4 *>(ap[nt] + (size_t)step * 32));
                        bf[nt][0][0] = __byte_perm(x.x, x.z, 0x5410);
                        bf[nt][0][1] = __byte_perm(x.x, x.z, 0x7632);
                        bf[nt][1][0] = __byte_perm(x.y, x.w, 0x5410);
                        bf[nt][1][1] = __byte_perm(x.y, x.w, 0x7632);
                    }
                    const uint32_t wc[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        const uint32_t lo = wc[2 * mt], hi = wc[2 * mt + 1];
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const uint32_t a0 = Deq<T>::sub(lop3_and_or(lo >> (8 * q), 0x000F000Fu, Deq<T>::kMagic), zc[2 * mt]);
                            const uint32_t a1 = Deq<T>::sub(lop3_and_or(hi >> (8 * q), 0x000F000Fu, Deq<T>::kMagic), zc[2 * mt + 1]);
                            const uint32_t a2 = Deq<T>::sub(lop3_and_or(lo >> (8 * q + 4), 0x000F000Fu, Deq<T>::kMagic), zc[2 * mt]);
                            const uint32_t a3 = Deq<T>::sub(lop3_and_or(hi >> (8 * q + 4), 0x000F000Fu, Deq<T>::kMagic), zc[2 * mt + 1]);
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt)
                                mma_16816<T>(gacc[mt][nt], a0, a1, a2, a3, bf[nt][q][0], bf[nt][q][1]);
                        }
                    }
                }
                const float sc[4] = {f16_bits_to_f((uint16_t)(sw[v].x & 0xFFFF)), f16_bits_to_f((uint16_t)(sw[v].x >> 16)),
                                     f16_bits_to_f((uint16_t)(sw[v].y & 0xFFFF)), f16_bits_to_f((uint16_t)(sw[v].y >> 16))};
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        facc[mt][nt][0] = fmaf(gacc[mt][nt][0], sc[2 * mt], facc[mt][nt][0]);
                        facc[mt][nt][1] = fmaf(gacc[mt][nt][1], sc[2 * mt], facc[mt][nt][1]);
                        facc[mt][nt][2] = fmaf(gacc[mt][nt][2], sc[2 * mt + 1], facc[mt][nt][2]);
                        facc[mt][nt][3] = fmaf(gacc[mt][nt][3], sc[2 * mt + 1], facc[mt][nt][3]);
                    }
            }
        }
    }

    // ---- K-split reduction across the W warps ----
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[(warp * NE + (mt * NT + nt) * 4 + i) * 32 + lane] = facc[mt][nt][i];
    __syncthreads();
    for (int idx = threadIdx.x; idx < NE * 32; idx += blockDim.x) {
        float v = 0.f;
        for (int w = 0; w < W; ++w) v += red[w * NE * 32 + idx];
        const int e = idx >> 5, l = idx & 31;
        const int mt = e / (NT * 4), nt = (e / 4) % NT, i = e & 3;
        const int col = blockIdx.y * 32 + 4 * (l >> 2) + 2 * mt + (i >> 1);
        const int tok = tok0 + nt * 8 + 2 * (l & 3) + (i & 1);
        if (tok < M) store_out(C, c_dtype, (size_t)tok * N + col, v);
    }
}

template <typename T, int NT, int GSTEPS>
static int launch_gemv_t(const T *a, const int32_t *qweight, const int32_t *qzeros,
                         const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs,
                         int zero_offset, cudaStream_t st) {
    constexpr int kBatch = GemvCfg<NT>::kBatch;
    const int nsm = num_sms();
    const int nchunk = N / 32;
    const int mblocks = (M + 8 * NT - 1) / (8 * NT);
    const int nvg = K / (32 * GSTEPS);
    const int vpg = gs / (32 * GSTEPS);
    // Warps per CTA (the K split): as many as keep the whole grid resident in
    // one wave at the register budget, with >= 1 batch of work per warp.
    const long warp_capacity = (long)nsm * (65536 / (GemvCfg<NT>::kMaxRegs * 32));
    int W = (int)(warp_capacity / ((long)nchunk * mblocks));
    const int max_by_work = (nvg * GSTEPS + kBatch - 1) / kBatch;  // batches of the whole K
    W = W < 1 ? 1 : W;
    W = W > kGemvMaxWarps ? kGemvMaxWarps : W;
    W = W > max_by_work ? max_by_work : W;
    const int vpw = (nvg + W - 1) / W;
    W = (nvg + vpw - 1) / vpw;  // no idle warps
    const size_t smem = (size_t)W * (2 * NT * 4) * 32 * sizeof(float);
    dim3 grid(mblocks, nchunk), block(32 * W);
    gptq_gemv_kernel<T, NT, GSTEPS><<<grid, block, smem, st>>>(a, qweight, qzeros, scales, c, c_dtype, M,
                                                               N, K, zero_offset, vpg, vpw);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

template <typename T, int NT>
static int launch_gemv_nt(const T *a, const int32_t *qweight, const int32_t *qzeros,
                          const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs,
                          int zero_offset, cudaStream_t st) {
    if (gs % 128 == 0) return launch_gemv_t<T, NT, 4>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, st);
    if (gs % 64 == 0) return launch_gemv_t<T, NT, 2>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, st);
    return launch_gemv_t<T, NT, 1>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, st);
}

template <typename T>
static int launch_gemv(const void *a, const int32_t *qweight, const int32_t *qzeros,
                       const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs,
                       int zero_offset, cudaStream_t st) {
    const T *ap = static_cast<const T *>(a);
    if (M <= 8) return launch_gemv_nt<T, 1>(ap, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, st);
    return launch_gemv_nt<T, 2>(ap, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, st);
}

// Where the register-batched kernel is the faster decode design (measured on B200 against the
// shared-ring TMA kernel over the BASELINE shapes and their tensor-parallel shards): with two
// token tiles (9..16 tokens) its 16 warps per CTA, each with its own batch of independent 16-byte
// loads, hide the doubled MMA work better, except on mid-sized layers that are neither wide nor
// small (5120 x 5120 ties, 8704 x 5120 loses); with one tile it wins only on small layers from
// 5 tokens.  W4_GPTQ_DECODE (a tuning override of the TMA kernel) turns this choice off.
bool prefer_register_gemv(int M, int N, int K) {
    if (std::getenv("W4_GPTQ_DECODE")) return false;
    const long long nk = (long long)N * K;
    if (M > 8) return nk < 24LL * 1024 * 1024 || N >= 12288;
    return M >= 5 && nk < 12LL * 1024 * 1024;
}

int gptq_gemv(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
              const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs,
              int zero_offset, void *sync, void *ws, size_t ws_bytes, cudaStream_t st) {
    // Prefill-sized token counts: the tcgen05 GEMM (gptq_prefill.cu).  Decode: the
    // register-batched kernel above where it is the faster design (prefer_register_gemv), else
    // the shared-ring TMA kernel (gptq_decode.cu); the register-batched kernel also runs for
    // shapes the TMA kernel does not take, and every such call is counted
    // (w4_decode_fallback_count).
    if (M >= kPrefillMinM) {
        const int rp = gptq_prefill(a, a_dtype, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, ws,
                                    ws_bytes, st);
        if (rp >= 0) return rp;
    }
    if (M < kPrefillMinM && prefer_register_gemv(M, N, K) && aligned(a, 16) && aligned(qweight, 16) &&
        aligned(scales, 8)) {
        if (a_dtype == W4_BF16)
            return launch_gemv<__nv_bfloat16>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, st);
        return launch_gemv<__half>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, st);
    }
    const int rc = gptq_gemv_decode(a, a_dtype, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, sync,
                                    ws, ws_bytes, nullptr, st);
    if (rc >= 0) return rc;
    note_decode_fallback();
    if (a_dtype == W4_BF16)
        return launch_gemv<__nv_bfloat16>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, st);
    return launch_gemv<__half>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, st);
}

// ---------------------------------------------------------------------------
// Reference-formula kernel (dpas_s4_gptq_sc.cpp:146-233 contract, host oracle
// :273-288).  One thread per output; the group partial is an exact s32 and the
// fp32 epilogue uses the reference's operation order without contraction, so
// the f16 result is bit-identical to the host oracle.
// ---------------------------------------------------------------------------
__global__ void gptq_s4a_kernel(const uint8_t *__restrict__ a, const uint8_t *__restrict__ b,
                                const float *__restrict__ a_scale,
                                const uint16_t *__restrict__ s, uint16_t *__restrict__ c,
                                int rows, int cols, int dk) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    const int r = blockIdx.y;
    if (col >= cols) return;
    const int ngrp = dk / 128;
    const uint8_t *arow = a + (size_t)r * (dk / 2);
    const float as = a_scale[r];
    float acc = 0.f;
    for (int g = 0; g < ngrp; ++g) {
        int32_t s32 = 0;
        for (int kk = 0; kk < 128; kk += 2) {
            const int k = g * 128 + kk;
            const uint32_t ab = arow[k / 2];
            const uint32_t bb = b[(size_t)(k / 2) * cols + col];
            const int a0 = ((int)(ab << 28)) >> 28, a1 = ((int)(ab << 24)) >> 28;
            const int b0 = ((int)(bb << 28)) >> 28, b1 = ((int)(bb << 24)) >> 28;
            s32 += a0 * b0 + a1 * b1;
        }
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn((float)s32, as), f16_bits_to_f(s[(size_t)g * cols + col])));
    }
    c[(size_t)r * cols + col] = __half_as_ushort(__float2half_rn(acc));
}

int gptq_s4a(const uint8_t *a, const uint8_t *b, const float *a_scale, const uint16_t *s,
             uint16_t *c, int rows, int cols, int dk, cudaStream_t st) {
    dim3 block(128), grid((cols + 127) / 128, rows);
    gptq_s4a_kernel<<<grid, block, 0, st>>>(a, b, a_scale, s, c, rows, cols, dk);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

}  // namespace w4
