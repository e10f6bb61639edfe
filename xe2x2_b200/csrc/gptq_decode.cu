// gptq_decode.cu -- GPTQ int4 decode GEMM (M <= 16) over one shared TMA ring per CTA (sm_100a).
//
// Contract (w4_gptq_gemm at decode sizes):
//   C[m,n] = sum_g s[g,n] * sum_{k in g} A[m,k] * (q[k,n] - z[g,n])
// with q / z the checkpoint codes as stored (qweight i32 [K/8,N], eight codes LSB-first along K;
// qzeros i32 [K/gs,N/8] LSB-first along N; kernels/nvfp4/gptq_s4_dump.py:61-73,106-114 of the
// reference) and the group-partial-then-scale structure of the reference decode kernel
// (kernels/esimd_dpas/dpas_s4_gptq_sc.cpp:178-218).
//
// Organisation.  A CTA owns BN = 32*CW output columns and a contiguous run of 128-k stages of
// K.  One producer warp streams every stage -- CW tensor-map boxes of 16 qweight rows x 32
// columns (128-byte swizzled), the stage's scale rows and zero rows -- into a ring of S stages
// (as deep as shared memory allows) that all CW consumer warps read; a stage is refilled once
// every consumer warp has arrived on its "empty" barrier.  Consumer warp cw owns tile columns
// [32cw, 32cw + 32).  When the column tiles are too few to fill the SMs, K is split over ks CTAs
// (grid z): each writes its fp32 partial tile to the caller's workspace, fences, and increments
// the tile's counter in the workspace's sync area; the CTA that arrives last sums the ks partials
// in z order (fixed summation order) and stores the tile, and its increment wraps the counter
// back to zero.  No CTA waits for another, so the grid may take any number of waves.  A stage is
// 128 k whatever the group size, so any number of groups (tensor-parallel shards with 5 or 17)
// runs here.
//
// Activations.  The producer bulk-copies the CTA's activation rows (its K range) into shared
// memory with its first copies; the consumers then rewrite them in place, per row and 128-k unit
// (one group when gs < 128), as f16 scaled by the power of two 2^e that puts the unit's absolute
// maximum in [2^14, 2^15), in the order the MMA fragments want, values at odd k divided by 16.
// Every bf16 or f16 value of at least 2^-28 times its unit's maximum is represented exactly.
// The same pass records, per unit and row, the sums of the stored values at even and odd k and
// 2^-e, which the unit's fp32 result is multiplied by.
//
// Math, per consumer lane (g = lane/4, t = lane%4) and 32-k step j of a stage: the lane loads
// the 16-byte chunk of columns 4*sigma(g)..+3 of qweight row 4j + t (eight k each).  Two
// m16n8k16 f16 tiles take columns (4s, 4s+1) and (4s+2, 4s+3) as MMA rows g and g+8 (swap-AB:
// weight columns are MMA rows, tokens MMA columns).  MMA q of the step takes the code pairs
// (2q, 2q+4) and (2q+1, 2q+5) of each word: one lop3 with the f16 magic 1024.0 turns the pair
// in mantissa bits 0-3 into 1024 + q (even k) and the pair in bits 4-7 into 1024 + 16q (odd k),
// so the MMA operand needs no subtraction and one shift serves all eight codes of a word.
// Against the activations (a at even k, a/16 at odd k) the MMA sums
//   1024 * (sum of stored values) + sum_k q_k a_k,
// so the accumulator of each unit starts at -1024 * (sum of stored values) - z * sum_k a_k 2^e
// (from the recorded sums) and ends at 2^e sum_k (q_k - z) a_k; it is scaled by the fp16 group
// scale and 2^-e when the unit ends.  Products are exact; only the fp32 sums round.  Any consistent relabelling
// of k is a legal dot product; the activations in shared memory carry the same relabelling.
//
// Every wait is bounded (tma_util.cuh): an expired wait sets a device status word that
// w4_check_device_status() reports and the warp stops consuming.  No copy uses multicast.
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "tma_util.cuh"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

static __device__ unsigned int g_dec_timeout;  // a bounded wait expired (sticky until read)

namespace dec {

constexpr int kMaxStages = 8;  // ring depth limit
constexpr int kRows = 16;      // qweight rows (of 8 k) per stage: 128 k
constexpr int kStageK = 128;   // k per stage

__host__ __device__ constexpr int al128(int x) { return (x + 127) & ~127; }

// Activation row pitch in shared memory: 256 bytes per stage plus 64, so the two token rows of
// a shared-load phase fall in different halves of the 128-byte bank window.
__host__ __device__ inline int act_pitch(int max_stages) { return max_stages * 256 + 64; }

// Shared-memory layout of one CTA (byte offsets from a 1024-aligned base), the same on host
// and device: S weight stages | S scale stages | S zero stages | 2S + 1 barriers, a flag and 16
// row maxima | per-unit terms [units][16 rows] (float4) | activations [rows][P] and one zero row.
struct Lay {
    int w_stage, sc_stage, zr_stage, sc, zr, bars, flag, corr, act, total;
    __host__ __device__ Lay(int CW, int SG, int S, int max_st, int rows) {
        const int BN = 32 * CW;
        w_stage = CW * kRows * 128;
        sc_stage = al128(SG * BN * 2);
        zr_stage = al128(SG * BN / 2);
        sc = S * w_stage;
        zr = sc + S * sc_stage;
        bars = zr + S * zr_stage;
        flag = bars + (2 * S + 1) * 8;
        corr = al128(flag + 4 + 16 * 4);
        act = al128(corr + max_st * SG * 16 * 16);
        total = act + (rows + 1) * act_pitch(max_st);  // the last row stays zero
        (void)BN;
    }
};

// Lane quad g reads 16-byte chunk sigma(g) = (0,4,1,5,2,6,3,7)[g] of a 128-byte row: with the
// 128-byte swizzle (chunk ^= row % 8) the 8 lanes of a shared-load phase hit 8 distinct bank
// groups.
__device__ __forceinline__ int sigma(int g) { return (g >> 1) | ((g & 1) << 2); }

__device__ __forceinline__ bool wait_dec(uint64_t *bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicExch(&g_dec_timeout, 1u);
    return false;
}
// Release a ring stage (release semantics: this warp's reads of the stage are ordered before
// the producer's next copy into it).
__device__ __forceinline__ void release_stage(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Power-of-two exponent e that puts amax * 2^e in [2^14, 2^15), clamped to [-126, 126]
// (0 for a zero or non-finite amax).
__device__ __forceinline__ int row_exp(float amax) {
    const int be = (int)((__float_as_uint(amax) >> 23) & 0xFF);
    if (amax == 0.f || be == 255) return 0;
    const int e = 141 - be;  // 14 - (be - 127)
    return e < -126 ? -126 : (e > 126 ? 126 : e);
}
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }

// (x & m) | o as one three-input logic op (lut 0xEA); written out because the plain expression
// with two immediate masks was compiled to more than one instruction.
__device__ __forceinline__ uint32_t and_or(uint32_t x, uint32_t m, uint32_t o) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(x), "r"(m), "r"(o));
    return d;
}

__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// CW consumer warps + 1 producer warp.  GSTEPS = 32-k steps per unit (gs / 32, at most 4); SG =
// 4 / GSTEPS units (scale rows) per stage (one row for gs >= 128, read as row stage * 128 / gs).
// nst: 128-k stages of K, split over the ks CTAs along grid z; max_st: the most stages any CTA of
// the split holds; S: ring depth.  bf16: activations are bf16 (else f16).  part / cnt (ks > 1):
// fp32 partials [ks][M][N] and the tile counters (zero on entry, left zero).  grp: the token rows
// of each expert (the maps' z coordinate); M: all rows; rows_alloc: token rows a CTA holds.
// Register cap: 112 per thread with one token tile (two 288-thread or three 160-thread CTAs per
// SM; 3-5 % faster than 80 at 5120 x 17408 and 5120 x 5120, M = 1..8), 128 with two.
template <int NT> constexpr int dec_regs() { return NT == 1 ? 112 : 128; }

template <int CW, int NT, int GSTEPS>
__global__ void __maxnreg__(dec_regs<NT>())
gptq_decode_kernel(const __grid_constant__ CUtensorMap qw_map, const __grid_constant__ CUtensorMap sc_map,
                   const __grid_constant__ CUtensorMap zr_map, const uint16_t *__restrict__ A, void *__restrict__ C,
                   int c_dtype, int M, int N, int K, int has_z, int zero_offset, int nst, int max_st, int gs, int S,
                   int bf16, int pre, float *__restrict__ part, unsigned int *__restrict__ cnt,
                   unsigned int *__restrict__ rowmax, const __grid_constant__ ExpertRows grp, int rows_alloc) {
    constexpr int SG = 4 / GSTEPS;
    constexpr int BN = 32 * CW;
    extern __shared__ uint8_t smem_dyn[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    const int ks = (int)gridDim.z;
    const Lay L(CW, SG, S, max_st, rows_alloc);
    uint64_t *full = reinterpret_cast<uint64_t *>(base + L.bars);
    uint64_t *empty = full + S;
    uint64_t *actb = empty + S;  // the activation rows have landed
    float4 *corr = reinterpret_cast<float4 *>(base + L.corr);
    uint8_t *act = base + L.act;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n0 = blockIdx.y * BN;
    const int ex = expert_of_block(grp, blockIdx.x);
    const int tok0 = grp.row0[ex] + ((int)blockIdx.x - grp.blk0[ex]) * 8 * NT;
    const int rows = min(8 * NT, grp.row0[ex + 1] - tok0);  // real token rows of this CTA
    const int sb = (int)(blockIdx.z * (unsigned)nst / (unsigned)ks);
    const int ns = (int)((blockIdx.z + 1) * (unsigned)nst / (unsigned)ks) - sb;  // stages of this CTA
    const int P = act_pitch(max_st);

    if (warp == CW && lane == 0) {
        // the descriptors' first use would otherwise wait for their fetch
        prefetch_tensormap(&qw_map);
        prefetch_tensormap(&sc_map);
        if (has_z) prefetch_tensormap(&zr_map);
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        mbar_init(actb, 1);
        fence_mbar_init();
    }
    __syncthreads();  // barriers initialised before anyone waits on them

    if (warp == CW) {  // ---------------- producer warp ----------------
        if (lane == 0) {
            const uint32_t tx = CW * kRows * 128 + SG * BN * 2 + (has_z ? SG * BN / 2 : 0);
            int s = 0;
            auto issue = [&](int it) {
                const int st = sb + it;
                const int srow = GSTEPS == 4 ? (st * kStageK) / gs : st * SG;  // first scale row
                mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
                for (int c = 0; c < CW; ++c)
                    tma_load_3d(base + s * L.w_stage + c * kRows * 128, &qw_map, n0 + 32 * c, st * kRows, ex,
                                &full[s]);
                tma_load_3d(base + L.sc + s * L.sc_stage, &sc_map, n0, srow, ex, &full[s]);
                if (has_z) tma_load_3d(base + L.zr + s * L.zr_stage, &zr_map, n0 / 8, srow, ex, &full[s]);
                s = s + 1 == S ? 0 : s + 1;
            };
            // pre: the weights of the first ring fill are requested before the previous kernel on
            // the stream has completed (static weights, W4_OVERLAP_STATIC_WEIGHTS)
            const int pf = pre ? min(ns, S) : 0;
            for (int it = 0; it < pf; ++it) issue(it);
            grid_dep_wait();
            // the activation rows of this CTA's K range (16-byte multiples: K % 8 == 0)
            {
                const int kb = sb * kStageK;
                const int kn = min(ns * kStageK, K - kb);
                mbar_arrive_expect_tx(actb, (uint32_t)(rows * kn * 2));
                for (int r = 0; r < rows; ++r)
                    bulk_load_1d(base + L.act + r * P, A + (size_t)(tok0 + r) * K + kb, (uint32_t)(kn * 2), actb);
            }
            for (int it = pf; it < ns; ++it) {
                if (it >= S && !wait_dec(&empty[s], (uint32_t)(((it / S) - 1) & 1))) break;
                issue(it);
            }
        }
        __syncwarp();
        grid_dep_launch();  // every copy is issued: the next kernel may be scheduled
        return;             // consumers wait for every copy this warp issued
    }

    // ---------------- consumer warps ----------------
    // Activation rows -> f16 MMA operands in place (see the file comment).  Octet o (eight k) of
    // a row sits at byte 16 o of the row, rewritten as the pairs (0,4) (1,5) (2,6) (3,7); k beyond
    // K reads as zero.  A (row, unit) task of UO octets is one group of UO lanes.
    if (!__all_sync(0xffffffffu, wait_dec(actb, 0))) {
        // the copies never landed: the status word is set; compute on whatever is there
    }
    {
        constexpr int UO = 16 / SG;  // octets per unit
        constexpr int TPW = 32 / UO;  // tasks per warp and pass
        const int units = ns * SG;
        const int kb = sb * kStageK;
        const int sub = lane % UO;
        for (int task0 = warp * TPW; task0 < rows * units; task0 += CW * TPW) {  // warp-uniform trip count
            const int task = task0 + lane / UO;
            const bool valid = task < rows * units;
            const int r = valid ? task / units : 0, u = valid ? task - (task / units) * units : 0;
            const int o = u * UO + sub;
            uint4 x = make_uint4(0, 0, 0, 0);
            if (valid && kb + o * 8 < K) x = *reinterpret_cast<const uint4 *>(act + r * P + o * 16);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
            float v[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (bf16) {
                    v[2 * i] = __uint_as_float(w[i] << 16);
                    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
                } else {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
                    v[2 * i] = f.x;
                    v[2 * i + 1] = f.y;
                }
            }
            float am = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
            for (int off = UO / 2; off; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
            const int e = row_exp(am);
            const float sc = exp2i(e), sc16 = exp2i(e - 4);
            __half h[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = __float2half_rn(v[i] * ((i & 1) ? sc16 : sc));  // exact
            float se = 0.f, so = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                se += __half2float(h[i]);
                so += __half2float(h[i + 1]);
            }
#pragma unroll
            for (int off = UO / 2; off; off >>= 1) {
                se += __shfl_xor_sync(0xffffffffu, se, off);
                so += __shfl_xor_sync(0xffffffffu, so, off);
            }
            if (valid) {
                uint4 p;
                p.x = pack_h2(h[0], h[4]);
                p.y = pack_h2(h[1], h[5]);
                p.z = pack_h2(h[2], h[6]);
                p.w = pack_h2(h[3], h[7]);
                *reinterpret_cast<uint4 *>(act + r * P + o * 16) = p;
                if (sub == 0) corr[u * 16 + r] = make_float4(-1024.f * (se + so), -(se + 16.f * so), exp2i(-e), 0.f);
            }
        }
    }
    for (int o = threadIdx.x; o < ns * (kStageK / 8); o += CW * 32)
        *reinterpret_cast<uint4 *>(act + rows_alloc * P + o * 16) = make_uint4(0, 0, 0, 0);  // the zero row
    unsigned int *rmax = reinterpret_cast<unsigned int *>(base + L.flag + 4);  // this CTA's row maxima
    if (rowmax && threadIdx.x < 16) rmax[threadIdx.x] = 0u;
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");  // consumers only

    const int cw = warp;
    const int g = lane >> 2, t = lane & 3, sg = sigma(g);
    const int colw = 32 * cw + 4 * sg;  // first of this lane's four tile columns
    // this lane's 16-byte chunk of qweight row 4j + t within its warp's box
    uint32_t roff[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int r = 4 * j + t;
        roff[j] = cw * kRows * 128 + r * 128 + ((sg ^ (r & 7)) << 4);
    }
    // activation octet offsets of token tile nt; rows past M read the zero row
    uint32_t aoff[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int r = nt * 8 + g;
        aoff[nt] = (r < rows ? r : rows_alloc) * P + t * 16;
    }
    const uint32_t zsh = 16 * (sg & 1);
    const float zadd = has_z ? (float)zero_offset : 0.f;

    float facc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) facc[a][b][i] = 0.f;

    int s = 0;
    uint32_t ph = 0;
    for (int it = 0; it < ns; ++it) {
        if (!__all_sync(0xffffffffu, wait_dec(&full[s], ph))) break;  // the warp still meets the others below
        const uint8_t *wst = base + s * L.w_stage;
        const uint8_t *scs = base + L.sc + s * L.sc_stage;
        const uint8_t *zrs = base + L.zr + s * L.zr_stage;
        const uint8_t *ast = act + it * 256;
#pragma unroll
        for (int v = 0; v < SG; ++v) {
            const int unit = it * SG + v;
            const uint2 sw = *reinterpret_cast<const uint2 *>(scs + v * BN * 2 + colw * 2);
            const uint32_t zw = has_z ? (*reinterpret_cast<const uint32_t *>(zrs + v * (BN / 2) + (colw >> 3) * 4) >> zsh)
                                      : 0x8888u;
            float zf[4];
#pragma unroll
            for (int c = 0; c < 4; ++c)
                zf[c] = __int_as_float(0x4B000000 | ((zw >> (4 * c)) & 15u)) - 8388608.f + zadd;  // exact
            // accumulators start at -1024 * sum - z * sum_k a_k 2^e of the unit, per (column, token)
            float acc[2][NT][4], inv[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float4 c0 = corr[unit * 16 + nt * 8 + 2 * t], c1 = corr[unit * 16 + nt * 8 + 2 * t + 1];
                inv[nt][0] = c0.z;
                inv[nt][1] = c1.z;
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    acc[mt][nt][0] = fmaf(zf[2 * mt], c0.y, c0.x);
                    acc[mt][nt][1] = fmaf(zf[2 * mt], c1.y, c1.x);
                    acc[mt][nt][2] = fmaf(zf[2 * mt + 1], c0.y, c0.x);
                    acc[mt][nt][3] = fmaf(zf[2 * mt + 1], c1.y, c1.x);
                }
            }
#pragma unroll
            for (int i = 0; i < GSTEPS; ++i) {
                const int j = v * GSTEPS + i;
                const uint4 wv = *reinterpret_cast<const uint4 *>(wst + roff[j]);
                uint4 xb[NT];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) xb[nt] = *reinterpret_cast<const uint4 *>(ast + aoff[nt] + j * 64);
                const uint32_t wc[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int q = 0; q < 2; ++q) {
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        const uint32_t w0 = wc[2 * mt] >> (8 * q), w1 = wc[2 * mt + 1] >> (8 * q);
                        const uint32_t a0 = and_or(w0, 0x000F000Fu, 0x64006400u);  // row g, even k
                        const uint32_t a2 = and_or(w0, 0x00F000F0u, 0x64006400u);  // row g, odd k
                        const uint32_t a1 = and_or(w1, 0x000F000Fu, 0x64006400u);  // row g + 8
                        const uint32_t a3 = and_or(w1, 0x00F000F0u, 0x64006400u);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
                            mma_16816<__half>(acc[mt][nt], a0, a1, a2, a3, q ? xb[nt].z : xb[nt].x,
                                              q ? xb[nt].w : xb[nt].y);
                    }
                }
            }
            const float2 s01 = __half22float2(*reinterpret_cast<const __half2 *>(&sw.x));
            const float2 s23 = __half22float2(*reinterpret_cast<const __half2 *>(&sw.y));
            const float scl[4] = {s01.x, s01.y, s23.x, s23.y};
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        facc[mt][nt][i] = fmaf(acc[mt][nt][i], scl[2 * mt + (i >> 1)] * inv[nt][i & 1], facc[mt][nt][i]);
        }
        __syncwarp();  // every lane is done with stage s
        if (lane == 0) release_stage(&empty[s]);
        if (++s == S) {
            s = 0;
            ph ^= 1u;
        }
    }
    grid_dep_launch();  // late trigger: the next grid's CTAs take the slots this one frees

    // ---- output: lane element (mt, nt, i) is column colw + 2mt + (i >> 1), token 8nt + 2t + (i & 1)
    if (ks == 1) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int tr = nt * 8 + 2 * t + (i & 1);
                    if (tr < rows) {
                        store_out(C, c_dtype, (size_t)(tok0 + tr) * N + n0 + colw + 2 * mt + (i >> 1), facc[mt][nt][i]);
                        if (rowmax) fold_rowmax(rmax, tr, facc[mt][nt][i]);
                    }
                }
        if (rowmax) publish_rowmax<CW>(rmax, rowmax + tok0, rows);
        return;
    }
    // K split: this CTA's partial tile -> part[z][token][column] (16-byte stores of four
    // columns), then the tile's counter; the last of the ks CTAs sums the partials in z order.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int tr = nt * 8 + 2 * t + i;
            if (tr < rows)
                *reinterpret_cast<float4 *>(part + ((size_t)blockIdx.z * M + tok0 + tr) * N + n0 + colw) =
                    make_float4(facc[0][nt][i], facc[0][nt][i + 2], facc[1][nt][i], facc[1][nt][i + 2]);
        }
    // Publish: the CTA barrier orders every consumer's partials before thread 0's count, whose
    // release (cumulative) publishes them at device scope; its acquire orders the other CTAs'
    // partials before this CTA's reads (the last one), which the second barrier passes on.
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
    int *flag = reinterpret_cast<int *>(base + L.flag);
    if (threadIdx.x == 0) {
        const unsigned int tile = blockIdx.x * gridDim.y + blockIdx.y;
        *flag = atom_inc_acq_rel(&cnt[tile], (unsigned int)(ks - 1)) == (unsigned int)(ks - 1);  // wraps to 0
    }
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
    if (!*flag) return;
    for (int q = threadIdx.x; q < rows * (BN / 4); q += CW * 32) {
        const int tr = q / (BN / 4), c4 = (q - tr * (BN / 4)) * 4;
        const size_t o = (size_t)(tok0 + tr) * N + n0 + c4;
        float4 v = __ldcg(reinterpret_cast<const float4 *>(part + o));
        for (int z = 1; z < ks; ++z) {
            const float4 u = __ldcg(reinterpret_cast<const float4 *>(part + (size_t)z * M * N + o));
            v.x += u.x, v.y += u.y, v.z += u.z, v.w += u.w;
        }
        store_out(C, c_dtype, o, v.x);
        store_out(C, c_dtype, o + 1, v.y);
        store_out(C, c_dtype, o + 2, v.z);
        store_out(C, c_dtype, o + 3, v.w);
        if (rowmax) fold_rowmax(rmax, tr, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    if (rowmax) publish_rowmax<CW>(rmax, rowmax + tok0, rows);
}

}  // namespace dec

// ---- host side ----
namespace {

struct DecChoice {
    int cw, ks, S;  // S = 0: as deep as the shared-memory budget allows
};

// Optional tile override for tuning sweeps: W4_GPTQ_DECODE="cw,ks[,S]" (cw in {1,2,4,8}, ks 1..8,
// S ring stages 2..8), or "reg" to decline every call (the register-streamed kernel runs).
bool env_decline() {
    const char *e = std::getenv("W4_GPTQ_DECODE");
    return e && e[0] == 'r';
}
bool env_choice(DecChoice &c) {
    const char *e = std::getenv("W4_GPTQ_DECODE");
    if (!e) return false;
    int cw = 0, ks = 0, S = 0;
    if (std::sscanf(e, "%d,%d,%d", &cw, &ks, &S) < 2) return false;
    if ((cw != 1 && cw != 2 && cw != 4 && cw != 8) || ks < 1 || ks > 8 || S < 0 || S == 1 || S > dec::kMaxStages)
        return false;
    c = {cw, ks, S};
    return true;
}

constexpr int kSmemPerSm = 228 * 1024;  // shared memory of one SM
constexpr int kSmemPerCta = 227 * 1024;

// Ring depth: stages until the CTAs an SM holds share its shared memory, within [3, kMaxStages].
int ring_depth(int cw, int sg, int max_st, int rows, int per_sm) {
    const dec::Lay l0(cw, sg, 0, max_st, rows);
    const int fixed = l0.total + 1024 + 1024;  // layout without stages, alignment slack, system reserve
    const int per_stage = dec::Lay(cw, sg, 1, max_st, rows).total - l0.total;
    const int S = (kSmemPerSm / per_sm - fixed) / per_stage;
    return S < 3 ? 3 : (S > dec::kMaxStages ? dec::kMaxStages : S);
}

// CTAs of 32 (cw + 1) threads an SM holds by threads, registers and shared memory (with a ring
// of at least 3 stages).
int ctas_per_sm(int cw, int NT, int sg, int max_st, int rows) {
    const int threads = 32 * (cw + 1);
    const int by_thr = 2048 / threads;
    const int by_reg = 65536 / (threads * (NT == 1 ? dec::dec_regs<1>() : dec::dec_regs<2>()));
    const int by_smem = kSmemPerSm / (dec::Lay(cw, sg, 3, max_st, rows).total + 2048);
    int r = by_thr < by_reg ? by_thr : by_reg;
    r = r < by_smem ? r : by_smem;
    return r < 1 ? 1 : (r > 32 ? 32 : r);
}

// Tile width and K split.  The grid should be about one wave of CTAs with equal work, so HBM
// bandwidth is shared evenly: the target is 1.8 CTAs per SM with one token tile, 0.9 with two,
// whose CTAs hold twice the registers.  The K split is at most 8 and at most one CTA per 128-k
// stage.  A 256-column tile is taken when its tiles, split, reach the target; else a 128-column
// tile when they reach a quarter of it; else 64, else 32 columns (narrow shards such as 896
// columns run fastest on 64-column tiles).  Then the smallest K split that reaches the target.
// Measured on 17408, 5120, 4352 and 896 columns with K from 640 to 8704.  mblocks: token blocks
// of the call (over all experts).
DecChoice choose(int mblocks, int N, int K, int NT) {
    DecChoice c{1, 1, 0};
    if (env_choice(c) && N % (32 * c.cw) == 0) return c;
    const int nsm = num_sms();
    const int nst = (K + dec::kStageK - 1) / dec::kStageK;
    const int ks_cap = nst > 8 ? 8 : nst;
    const long target = NT == 1 ? (long)(1.8 * nsm) : (long)(0.9 * nsm);
    const int cws[4] = {8, 4, 2, 1};
    const long need[4] = {target, target / 4, 0, 0};
    for (int i = 0; i < 4; ++i) {
        const int cw = cws[i];
        if (N % (32 * cw)) continue;
        const long tiles = (long)(N / (32 * cw)) * mblocks;
        if (tiles * ks_cap < need[i]) continue;  // too few tiles: a narrower one
        int ks = 1;
        while (ks < ks_cap && tiles * ks < target) ++ks;
        return {cw, ks, 0};
    }
    return c;
}

// One decode GEMM call: E stacked weight matrices, grp.n expert row groups (1 for a plain GEMM).
struct DecCall {
    const void *a;
    int a_dtype;
    const int32_t *qweight, *qzeros;
    const uint16_t *scales;
    void *c;
    int c_dtype, M, N, K, gs, zero_offset, E, NT, rows_alloc;
    ExpertRows grp;
    unsigned int *cnt, *rowmax;
    float *part;
};

}  // namespace

template <int CW, int NT, int GSTEPS>
static int launch_dec_t(const DecCall &q, DecChoice ch, cudaStream_t st) {
    constexpr int SG = 4 / GSTEPS;
    constexpr int BN = 32 * CW;
    const int N = q.N, K = q.K, gs = q.gs;
    const int nst = (K + dec::kStageK - 1) / dec::kStageK;
    const int ks = ch.ks > nst ? nst : ch.ks;
    const int max_st = (nst + ks - 1) / ks;
    const int mblocks = q.grp.blk0[q.grp.n];
    const int rows = q.rows_alloc;
    if (mblocks == 0) return W4_OK;  // no token rows
    int S = ch.S;
    if (S == 0) {
        // the CTAs an SM will hold: its limit, or fewer when the grid is smaller than a wave
        const long grid_ctas = (long)mblocks * (N / BN) * ks;
        const int nsm = num_sms();
        int per_sm = ctas_per_sm(CW, NT, SG, max_st, rows);
        const int fill = (int)((grid_ctas + nsm - 1) / nsm);
        if (fill < per_sm) per_sm = fill;
        S = ring_depth(CW, SG, max_st, rows, per_sm);
    }
    const size_t smem = 1024 + (size_t)dec::Lay(CW, SG, S, max_st, rows).total;
    if (smem > (size_t)kSmemPerCta) return -1;
    const uint64_t E = (uint64_t)q.E, ng = (uint64_t)(K / gs);
    CUtensorMap qw_map, sc_map, zr_map;
    if (!make_map_3d(&qw_map, CU_TENSOR_MAP_DATA_TYPE_INT32, q.qweight, N, K / 8, E, (uint64_t)N * 4,
                     (uint64_t)(K / 8) * N * 4, 32, dec::kRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_3d(&sc_map, CU_TENSOR_MAP_DATA_TYPE_UINT16, q.scales, N, ng, E, (uint64_t)N * 2, ng * N * 2, BN, SG,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return -1;
    const int has_z = q.qzeros != nullptr;
    if (has_z) {
        if (!make_map_3d(&zr_map, CU_TENSOR_MAP_DATA_TYPE_INT32, q.qzeros, N / 8, ng, E, (uint64_t)N / 2,
                         ng * N / 2, BN / 8, SG, CU_TENSOR_MAP_SWIZZLE_NONE))
            return -1;
    } else {
        zr_map = sc_map;  // unused
    }
    auto kern = dec::gptq_decode_kernel<CW, NT, GSTEPS>;
    {
        static std::mutex mu;
        static bool set_dev[128] = {};
        int dev = 0;
        W4_CUDA_TRY(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lk(mu);
        if (dev < 0 || dev >= 128 || !set_dev[dev]) {
            W4_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemPerCta));
            W4_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
            if (dev >= 0 && dev < 128) set_dev[dev] = true;
        }
    }
    // static weights: the first ring fill is requested before the previous kernel completes, for
    // at most four token rows on layers of at most 16 MB of codes (measured faster there: 5120^2
    // M=1; slower on wider layers, where the early copies compete with the draining kernel's,
    // and at 8 rows)
    const int pre = launch_overlap() == W4_OVERLAP_STATIC_WEIGHTS && q.rows_alloc <= 4 &&
                    (long long)N * K / 2 * q.E <= (16LL << 20);
    dim3 grid(mblocks, N / BN, ks), block(32 * (CW + 1));
    W4_CUDA_TRY(launch_decode(kern, grid, block, smem, st, 1u, qw_map, sc_map, zr_map,
                              static_cast<const uint16_t *>(q.a), q.c, q.c_dtype, q.M, N, K, has_z, q.zero_offset, nst,
                              max_st, gs, S, (int)(q.a_dtype == W4_BF16), pre, q.part, q.cnt, q.rowmax, q.grp,
                              q.rows_alloc));
    return W4_OK;
}

template <int CW, int NT>
static int launch_dec_g(const DecCall &q, DecChoice ch, cudaStream_t st) {
    if (q.gs % 128 == 0) return launch_dec_t<CW, NT, 4>(q, ch, st);
    if (q.gs == 64) return launch_dec_t<CW, NT, 2>(q, ch, st);
    if (q.gs == 32) return launch_dec_t<CW, NT, 1>(q, ch, st);
    return -1;
}

template <int NT>
static int launch_dec_nt(const DecCall &q, DecChoice ch, cudaStream_t st) {
    switch (ch.cw) {
        case 8: return launch_dec_g<8, NT>(q, ch, st);
        case 4: return launch_dec_g<4, NT>(q, ch, st);
        case 2: return launch_dec_g<2, NT>(q, ch, st);
        case 1: return launch_dec_g<1, NT>(q, ch, st);
        default: return -1;
    }
}

static bool decode_shape_ok(int N, int K, int gs) {
    return N % 32 == 0 && K % 8 == 0 && K % gs == 0 && (gs % 128 == 0 || gs == 64 || gs == 32);
}

// The most rows of any expert of a call, and the checks of its offsets (off[0] = 0, nondecreasing).
static int max_rows(const int *off, int n) {
    if (!off || n < 1 || n > kMaxExperts || off[0] != 0) return -1;
    int m = 0;
    for (int e = 0; e < n; ++e) {
        if (off[e + 1] < off[e]) return -1;
        m = off[e + 1] - off[e] > m ? off[e + 1] - off[e] : m;
    }
    return m;
}

// The K-split partials a call takes (0: unsplit), for experts with row offsets off[0..n].
static size_t split_bytes_for(const int *off, int n, int N, int K, int gs) {
    const int mr = max_rows(off, n);
    if (mr < 0 || !decode_shape_ok(N, K, gs)) return 0;
    const int NT = mr <= 8 ? 1 : 2;
    ExpertRows g;
    if (!expert_rows(g, off, n, 8 * NT)) return 0;
    const DecChoice ch = choose(g.blk0[n], N, K, NT);
    const int nst = (K + dec::kStageK - 1) / dec::kStageK;
    const int ks = ch.ks > nst ? nst : ch.ks;
    return ks > 1 ? (size_t)ks * off[n] * N * 4 : 0;
}

size_t gptq_decode_split_bytes(int M, int N, int K, int gs) {
    if (M < 1 || M > 16) return 0;
    const int off[2] = {0, M};
    return split_bytes_for(off, 1, N, K, gs);
}

size_t gptq_decode_grouped_split_bytes(const int *off, int n, int N, int K, int gs) {
    return split_bytes_for(off, n, N, K, gs);
}

static int run_decode(DecCall &q, const int *off, int n, void *sync, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (env_decline()) return -1;
    const int mr = max_rows(off, n);
    if (mr < 0 || !decode_shape_ok(q.N, q.K, q.gs)) return -1;
    if (!aligned(q.qweight, 16) || !aligned(q.scales, 16) || (q.qzeros && !aligned(q.qzeros, 16)) || !aligned(q.a, 16))
        return -1;
    q.NT = mr <= 8 ? 1 : 2;
    q.rows_alloc = mr < 8 * q.NT ? mr : 8 * q.NT;
    q.M = off[n];
    if (!expert_rows(q.grp, off, n, 8 * q.NT)) return -1;
    if (q.M == 0) return W4_OK;
    DecChoice ch = choose(q.grp.blk0[n], q.N, q.K, q.NT);
    const int nst = (q.K + dec::kStageK - 1) / dec::kStageK;
    if (ch.ks > nst) ch.ks = nst;
    const long tiles = (long)(q.N / (32 * ch.cw)) * q.grp.blk0[n];
    // The K split needs the workspace: fp32 partials and one counter per tile in the sync area.
    if (ch.ks > 1 && (!sync || !ws || !aligned(ws, 16) || ws_bytes < (size_t)ch.ks * q.M * q.N * 4 ||
                      tiles > (long)kSyncTileCounters))
        ch.ks = 1;
    q.cnt = static_cast<unsigned int *>(sync);
    q.part = static_cast<float *>(ws);
    if (q.NT == 1) return launch_dec_nt<1>(q, ch, st);
    return launch_dec_nt<2>(q, ch, st);
}

int gptq_gemv_decode(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                     const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset,
                     void *sync, void *ws, size_t ws_bytes, unsigned int *rowmax, cudaStream_t st) {
    if (M < 1 || M > 16) return -1;
    DecCall q{};
    q.a = a, q.a_dtype = a_dtype, q.qweight = qweight, q.qzeros = qzeros, q.scales = scales, q.c = c;
    q.c_dtype = c_dtype, q.N = N, q.K = K, q.gs = gs, q.zero_offset = zero_offset, q.E = 1, q.rowmax = rowmax;
    const int off[2] = {0, M};
    return run_decode(q, off, 1, sync, ws, ws_bytes, st);
}

int gptq_gemv_decode_grouped(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                             const uint16_t *scales, const int *off, int n, void *c, int c_dtype, int N, int K, int gs,
                             int zero_offset, void *sync, void *ws, size_t ws_bytes, cudaStream_t st) {
    DecCall q{};
    q.a = a, q.a_dtype = a_dtype, q.qweight = qweight, q.qzeros = qzeros, q.scales = scales, q.c = c;
    q.c_dtype = c_dtype, q.N = N, q.K = K, q.gs = gs, q.zero_offset = zero_offset, q.E = n, q.rowmax = nullptr;
    return run_decode(q, off, n, sync, ws, ws_bytes, st);
}

int take_decode_wait_status() {
    unsigned int v = 0;
    W4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_dec_timeout, sizeof(v)));
    if (v) {
        const unsigned int zero = 0;
        W4_CUDA_TRY(cudaMemcpyToSymbol(g_dec_timeout, &zero, sizeof(zero)));
        set_error("a device-side wait expired in the GPTQ decode GEMM");
        return W4_ERR_TIMEOUT;
    }
    return W4_OK;
}

}  // namespace w4
