// nvfp4_decode.cu -- NVFP4 W4A16 decode GEMM over one shared TMA ring per CTA (sm_100a).
//
// Contract: w4_nvfp4_gemm with act_mode W4A16 on the K-contiguous layout and E4M3 block scales,
//   C[m,n] = (sum_k A[m,k] * (e2m1(w[n,k]) * s[k/16,n])) * global
// (the external operator nvfp4_gemm_w4a16[_f8scale], kernels/nvfp4/bench_nvfp4_m1.py:67,88;
// the reference LUT kernel's host loop kernels/nvfp4/nibble_lut_sc.cpp:319-330 without the
// block scales).
//
// Organisation (as the GPTQ decode GEMM, gptq_decode.cu).  A CTA owns BN = 32*CW output columns,
// 8*NT tokens and a contiguous run of 256-k stages of K.  One producer warp first bulk-copies
// the CTA's activation rows (its K range), then streams every stage -- CW tensor-map boxes of 32
// weight rows x 128 bytes of [N, K/2] (128-byte swizzled) and the stage's 16 x BN block scales
// -- into a ring of S stages that all CW consumer warps read; a stage is refilled once every
// consumer warp has arrived on its "empty" barrier.  Consumer warp cw owns tile columns
// [32cw, 32cw + 32).  When the column tiles are too few to fill the SMs, K is split over ks CTAs
// (grid z): each writes its fp32 partial tile to the caller's workspace and counts itself on the
// tile's counter in the workspace's sync area; the CTA that arrives last sums the ks partials in
// z order (fixed summation order) and stores the tile, and its increment wraps the counter back
// to zero.  No CTA waits for another.
//
// Activations.  The consumers rewrite the bf16 rows in place, per row and 128-k unit, as f16
// scaled by the power of two 2^e that puts the unit's absolute maximum in [2^14, 2^15) (exact for
// every value of at least 2^-28 times the unit's maximum), and record 2^-e per unit and row.  The
// unit's sixteen 8-k chunks are stored permuted (chunk 4t + q at position 4q + (t + q) % 4) so
// that the 128-bit loads of a quarter-warp (two rows x four lanes) hit eight distinct bank groups.
//
// Math (f16 warp MMA, swap-AB: weight columns are MMA rows, tokens MMA columns): lane (g = lane/4,
// t = lane%4) owns the weight columns 32cw + 4g + c (c = 0..3: m-tile 0 rows g / g+8 are columns
// 4g / 4g+1, m-tile 1 columns 4g+2 / 4g+3) and k 32t..32t+31 of each unit, so its block scales of
// a 16-k block are four consecutive bytes.  MMA step j covers k = 32t + 4j .. +3 of the lane
// (operand slots 2t, 2t+1 <- +0, +1 and 2t+8, 2t+9 <- +2, +3): one byte of codes is one
// hardware e2m1x2 -> f16x2 conversion, multiplied by the f16 block scale (e4m3 -> f16 is exact,
// and e2m1 * e4m3 has at most 6 significant bits and lies in [2^-10, 2688], so the product is an
// exact f16).  Products in the MMA are exact; only the fp32 sums round.  Each unit's sum is
// scaled by 2^-e into the result and the tensor scale multiplies the final sum.
//
// Every wait is bounded (tma_util.cuh): an expired wait sets a device status word that
// w4_check_device_status() reports and the warp stops consuming.  No copy uses multicast.
#include <cuda_fp8.h>

#include <cstdlib>
#include <mutex>

#include "tma_util.cuh"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

static __device__ unsigned int g_fp4d_timeout;  // a bounded wait expired (sticky until read)

namespace fp4d {

constexpr int kMaxStages = 8;  // ring depth limit
constexpr int KS = 256;        // k per stage (two 128-k units)

__host__ __device__ constexpr int al128(int x) { return (x + 127) & ~127; }

// Activation row pitch in shared memory: 512 bytes per stage plus 64, so consecutive token rows
// fall in different halves of the 128-byte bank window.
__host__ __device__ inline int act_pitch(int max_st) { return max_st * 512 + 64; }

// Shared-memory layout of one CTA (byte offsets from a 1024-aligned base), the same on host and
// device: S weight stages (CW boxes of 4 KB) | S scale stages (16 x BN E4M3) | 2S + 1 barriers,
// a flag and 16 row maxima | 2^-e [units][16 rows] | activations [rows][P] and one zero row.
struct Lay {
    int w_stage, s_stage, sc, bars, flag, inv, act, total;
    __host__ __device__ Lay(int CW, int S, int max_st, int rows) {
        w_stage = CW * 32 * 128;
        s_stage = al128(16 * 32 * CW);
        sc = S * w_stage;
        bars = sc + S * s_stage;
        flag = bars + (2 * S + 1) * 8;
        inv = al128(flag + 4 + 16 * 4);
        act = al128(inv + max_st * 2 * 16 * 4);
        total = act + (rows + 1) * act_pitch(max_st);
    }
};

__device__ __forceinline__ bool wait_fp4d(uint64_t *bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicExch(&g_fp4d_timeout, 1u);
    return false;
}

// Exponent e that puts amax * 2^e in [2^14, 2^15), clamped to [-126, 126] (0 for a zero or
// non-finite amax).
__device__ __forceinline__ int unit_exp(float amax) {
    const int be = (int)((__float_as_uint(amax) >> 23) & 0xFF);
    if (amax == 0.f || be == 255) return 0;
    const int e = 141 - be;  // 14 - (be - 127)
    return e < -126 ? -126 : (e > 126 ? 126 : e);
}
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }

// The two E2M1 codes of byte `sel` of w (low nibble first) as f16x2, by the hardware conversion.
template <int SEL> __device__ __forceinline__ uint32_t e2m1x2_f16(uint32_t w) {
    uint32_t r;
    asm("{\n.reg .b8 b0, b1, b2, b3;\nmov.b32 {b0, b1, b2, b3}, %1;\ncvt.rn.f16x2.e2m1x2 %0, b" "%2" ";\n}"
        : "=r"(r)
        : "r"(w), "n"(SEL));
    return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// Four E4M3 block scales (columns 4g + c, c = 0..3) -> f16 pairs broadcast to both halves.
__device__ __forceinline__ void load_scales4(const uint8_t *p, uint32_t (&sc)[4]) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
    const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xFFFFu), __NV_E4M3);
    const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3);
    const uint32_t l = (uint32_t)lo.x | ((uint32_t)lo.y << 16), h = (uint32_t)hi.x | ((uint32_t)hi.y << 16);
    sc[0] = __byte_perm(l, 0, 0x1010);
    sc[1] = __byte_perm(l, 0, 0x3232);
    sc[2] = __byte_perm(h, 0, 0x1010);
    sc[3] = __byte_perm(h, 0, 0x3232);
}

// Register cap per thread: 128 with one token tile, 168 with two.
template <int NT> constexpr int fp4d_regs() { return NT == 1 ? 128 : 168; }

// CW consumer warps + 1 producer warp.  nst: 256-k stages of K, split over the ks CTAs along grid
// z; max_st: the most stages any CTA of the split holds; S: ring depth.  part / cnt (ks > 1):
// fp32 partials [ks][M][N] and the tile counters (zero on entry, left zero).
template <int CW, int NT>
__global__ void __maxnreg__((fp4d_regs<NT>()))
nvfp4_decode_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap sc_map,
                    const uint16_t *__restrict__ A, const float *__restrict__ global_scale, void *__restrict__ C,
                    int c_dtype, int M, int N, int K, int nst, int max_st, int S, int pre, int rows_alloc,
                    const __grid_constant__ ExpertRows grp,
                    float *__restrict__ part, unsigned int *__restrict__ cnt, unsigned int *__restrict__ rowmax) {
    constexpr int BN = 32 * CW;
    extern __shared__ uint8_t smem_dyn[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    const Lay L(CW, S, max_st, rows_alloc);
    uint64_t *full = reinterpret_cast<uint64_t *>(base + L.bars);
    uint64_t *empty = full + S;
    uint64_t *actb = empty + S;  // the activation rows have landed
    float *inv = reinterpret_cast<float *>(base + L.inv);
    uint8_t *act = base + L.act;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ex = expert_of_block(grp, blockIdx.x);
    const int tok0 = grp.row0[ex] + ((int)blockIdx.x - grp.blk0[ex]) * 8 * NT;
    const int rows = min(8 * NT, grp.row0[ex + 1] - tok0);  // real token rows of this CTA
    const int n0 = blockIdx.y * BN;
    const int ks = (int)gridDim.z;
    const int sb = (int)(blockIdx.z * (unsigned)nst / (unsigned)ks);
    const int ns = (int)((blockIdx.z + 1) * (unsigned)nst / (unsigned)ks) - sb;  // stages of this CTA
    const int P = act_pitch(max_st);

    if (warp == CW && lane == 0) {
        // the descriptors' first use would otherwise wait for their fetch
        prefetch_tensormap(&w_map);
        prefetch_tensormap(&sc_map);
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
            const uint32_t tx = CW * 32 * 128 + 16 * BN;
            int s = 0, wraps = 0;
            auto issue = [&](int it) {
                const int st = sb + it;
                mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
                for (int c = 0; c < CW; ++c)
                    tma_load_3d(base + s * L.w_stage + c * 32 * 128, &w_map, st * (KS / 2), n0 + 32 * c, ex,
                                &full[s]);
                tma_load_3d(base + L.sc + s * L.s_stage, &sc_map, n0, st * (KS / 16), ex, &full[s]);
                if (++s == S) {
                    s = 0;
                    ++wraps;
                }
            };
            // pre: codes and block scales of the first ring fill are requested before the previous
            // kernel on the stream has completed (static weights, W4_OVERLAP_STATIC_WEIGHTS)
            const int pf = pre ? min(ns, S) : 0;
            for (int it = 0; it < pf; ++it) issue(it);
            grid_dep_wait();  // activations are the previous kernel's output
            // the activation rows of this CTA's K range (16-byte multiples: K % 128 == 0)
            {
                const int kb = sb * KS;
                const int kn = min(ns * KS, K - kb);
                mbar_arrive_expect_tx(actb, (uint32_t)(rows * kn * 2));
                for (int r = 0; r < rows; ++r)
                    bulk_load_1d(act + r * P, A + (size_t)(tok0 + r) * K + kb, (uint32_t)(kn * 2), actb);
            }
            for (int it = pf; it < ns; ++it) {
                if (it >= S && !wait_fp4d(&empty[s], (uint32_t)((wraps - 1) & 1))) break;  // wraps = it / S
                issue(it);
            }
        }
        __syncwarp();
        grid_dep_launch();  // every copy is issued: the next kernel may be scheduled
        return;             // consumers wait for every copy this warp issued
    }

    // ---------------- consumer warps ----------------
    if (!__all_sync(0xffffffffu, wait_fp4d(actb, 0))) {
        // the copies never landed: the status word is set; compute on whatever is there
    }
    {
        // Activations -> f16 in place.  A task is one (row, 128-k unit): a group of 16 lanes, one
        // 8-k chunk each.  k beyond K reads as zero.
        const int units = 2 * ns;
        const int kb = sb * KS;
        const int sub = lane & 15;
        const int tq = sub >> 2, qq = sub & 3;
        const int dst = 4 * qq + ((tq + qq) & 3);  // the chunk's permuted position
        for (int task0 = warp * 2; task0 < rows * units; task0 += CW * 2) {  // warp-uniform trip count
            const int task = task0 + (lane >> 4);
            const bool valid = task < rows * units;
            const int r = valid ? task / units : 0, u = valid ? task - (task / units) * units : 0;
            uint8_t *ub = act + r * P + u * 256;
            uint4 x = make_uint4(0, 0, 0, 0);
            if (valid && kb + u * 128 + sub * 8 < K) x = *reinterpret_cast<const uint4 *>(ub + sub * 16);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
            float v[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[2 * i] = __uint_as_float(w[i] << 16);
                v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
            }
            float am = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
            for (int off = 8; off; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
            const int e = unit_exp(am);
            const float scl = exp2i(e);
            uint4 h;
            uint32_t *hw = reinterpret_cast<uint32_t *>(&h);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __half2 p = __floats2half2_rn(v[2 * i] * scl, v[2 * i + 1] * scl);  // exact
                hw[i] = *reinterpret_cast<const uint32_t *>(&p);
            }
            __syncwarp();  // every chunk of the unit is read before any is overwritten
            if (valid) {
                *reinterpret_cast<uint4 *>(ub + dst * 16) = h;
                if (sub == 0) inv[u * 16 + r] = exp2i(-e);
            }
        }
        for (int o = threadIdx.x; o < ns * (KS / 8); o += CW * 32)
            *reinterpret_cast<uint4 *>(act + rows_alloc * P + o * 16) = make_uint4(0, 0, 0, 0);  // the zero row
    }
    unsigned int *rmax = reinterpret_cast<unsigned int *>(base + L.flag + 4);  // this CTA's row maxima
    if (rowmax && threadIdx.x < 16) rmax[threadIdx.x] = 0u;
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");  // consumers only

    const int cw = warp;
    const int g = lane >> 2, t = lane & 3;
    // weights: row 4g + c of this warp's box, 16-byte chunk 4h + t of unit h, swizzled by row % 8
    uint32_t woff[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int r = 4 * g + c;
            woff[h][c] = cw * 32 * 128 + r * 128 + (((4 * h + t) ^ (r & 7)) << 4);
        }
    // activations: token row 8nt + g (the zero row past the CTA's rows), chunk 4t + q of a unit at
    // its permuted position
    uint32_t aoff[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int r = nt * 8 + g;
#pragma unroll
        for (int q = 0; q < 4; ++q) aoff[nt][q] = (r < rows ? r : rows_alloc) * P + (4 * q + ((t + q) & 3)) * 16;
    }
    const int colw = 32 * cw + 4 * g;  // first of this lane's four tile columns

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
        if (!__all_sync(0xffffffffu, wait_fp4d(&full[s], ph))) break;  // the warp still meets the others below
        const uint8_t *wst = base + s * L.w_stage;
        const uint8_t *sst = base + L.sc + s * L.s_stage;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int u = 2 * it + h;
            const uint8_t *ast = act + u * 256;
            uint4 wv[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) wv[c] = *reinterpret_cast<const uint4 *>(wst + woff[h][c]);
            uint32_t sc[2][4];
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) load_scales4(sst + (8 * h + 2 * t + hb) * BN + colw, sc[hb]);
            float acc[2][NT][4];
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int b = 0; b < NT; ++b)
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[a][b][i] = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 xa[NT];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) xa[nt] = *reinterpret_cast<const uint4 *>(ast + aoff[nt][q]);
                const int hb = q >> 1;
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    uint32_t a01[4], a23[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t word = q == 0 ? wv[c].x : q == 1 ? wv[c].y : q == 2 ? wv[c].z : wv[c].w;
                        const uint32_t lo = jj ? e2m1x2_f16<2>(word) : e2m1x2_f16<0>(word);
                        const uint32_t hi = jj ? e2m1x2_f16<3>(word) : e2m1x2_f16<1>(word);
                        a01[c] = hmul2(lo, sc[hb][c]);
                        a23[c] = hmul2(hi, sc[hb][c]);
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const uint32_t b0 = jj ? xa[nt].z : xa[nt].x, b1 = jj ? xa[nt].w : xa[nt].y;
                        mma_16816<__half>(acc[0][nt], a01[0], a01[1], a23[0], a23[1], b0, b1);
                        mma_16816<__half>(acc[1][nt], a01[2], a01[3], a23[2], a23[3], b0, b1);
                    }
                }
            }
            // unit end: the token's 2^-e
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float2 iv = *reinterpret_cast<const float2 *>(inv + u * 16 + nt * 8 + 2 * t);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) facc[mt][nt][i] = fmaf(acc[mt][nt][i], (i & 1) ? iv.y : iv.x, facc[mt][nt][i]);
            }
        }
        __syncwarp();  // every lane is done with stage s
        if (lane == 0)
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[s])) : "memory");
        if (++s == S) {
            s = 0;
            ph ^= 1u;
        }
    }
    grid_dep_launch();  // late trigger: the next grid's CTAs take the slots this one frees

    // ---- output: lane element (mt, nt, i) is column colw + 2mt + (i >> 1), token 8nt + 2t + (i & 1)
    const float gsc = global_scale ? global_scale[ex] : 1.0f;
    if (ks == 1) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int tr = nt * 8 + 2 * t + (i & 1);
                    if (tr < rows) {
                        const float v = facc[mt][nt][i] * gsc;
                        store_out(C, c_dtype, (size_t)(tok0 + tr) * N + n0 + colw + 2 * mt + (i >> 1), v);
                        if (rowmax) fold_rowmax(rmax, tr, v);
                    }
                }
        if (rowmax) publish_rowmax<CW>(rmax, rowmax + tok0, rows);
        return;
    }
    // K split: this CTA's partial tile -> part[z][token][column] (8-byte stores of two columns),
    // then the tile's counter; the last of the ks CTAs sums the partials in z order.
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int tr = nt * 8 + 2 * t + i;
                if (tr < rows)
                    *reinterpret_cast<float2 *>(part + ((size_t)blockIdx.z * M + tok0 + tr) * N + n0 + colw + 2 * mt) =
                        make_float2(facc[mt][nt][i], facc[mt][nt][i + 2]);
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
        v.x *= gsc, v.y *= gsc, v.z *= gsc, v.w *= gsc;
        store_out(C, c_dtype, o, v.x);
        store_out(C, c_dtype, o + 1, v.y);
        store_out(C, c_dtype, o + 2, v.z);
        store_out(C, c_dtype, o + 3, v.w);
        if (rowmax) fold_rowmax(rmax, tr, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    if (rowmax) publish_rowmax<CW>(rmax, rowmax + tok0, rows);
}

}  // namespace fp4d

// ---- host side ----
namespace {

struct Fp4Choice {
    int cw, ks, S;  // S = 0: as deep as the shared-memory budget allows
};

// Optional override for tuning sweeps: W4_NVFP4_DECODE="cw,ks[,S]" (cw in {1,2,4,8}, ks 1..8, S
// ring stages 2..8).
bool env_fp4_choice(Fp4Choice &c) {
    const char *e = std::getenv("W4_NVFP4_DECODE");
    if (!e) return false;
    int cw = 0, ks = 0, S = 0;
    if (std::sscanf(e, "%d,%d,%d", &cw, &ks, &S) < 2) return false;
    if ((cw != 1 && cw != 2 && cw != 4 && cw != 8) || ks < 1 || ks > 8 || S < 0 || S == 1 ||
        S > fp4d::kMaxStages)
        return false;
    c = {cw, ks, S};
    return true;
}

constexpr int kSmemPerSm = 228 * 1024;
constexpr int kSmemPerCta = 227 * 1024;

int fp4_regs(int NT) { return NT == 1 ? fp4d::fp4d_regs<1>() : fp4d::fp4d_regs<2>(); }

// CTAs of 32 (cw + 1) threads an SM holds by threads, registers and shared memory (3-stage ring).
int fp4_ctas_per_sm(int cw, int NT, int max_st, int rows) {
    const int threads = 32 * (cw + 1);
    const int by_thr = 2048 / threads;
    const int by_reg = 65536 / (threads * fp4_regs(NT));
    const int by_smem = kSmemPerSm / (fp4d::Lay(cw, 3, max_st, rows).total + 2048);
    int r = by_thr < by_reg ? by_thr : by_reg;
    r = r < by_smem ? r : by_smem;
    return r < 1 ? 1 : (r > 32 ? 32 : r);
}

// Tile width and K split.  The 128-column tile (four consumer warps) is taken whenever N allows
// it (measured faster than 256, 64 and 32 columns at every decode shape, small shards included),
// then the smallest K split, at most 8 and at most one CTA per 256-k stage, that reaches 1.3 CTAs
// per SM.  Measured on 5120 x 5120, 5120 x 17408, 640 x 5120, 2176 x 5120 and 1408 x 4096 at one
// and eight rows, the best split always gave 1.35 to 1.9 CTAs per SM; beyond one wave (three
// 160-thread CTAs of this kernel per SM) the call slows by a third.  mblocks: token blocks of the
// call (over all experts).
Fp4Choice fp4_choose(int mblocks, int N, int K) {
    Fp4Choice c{1, 1, 0};
    if (env_fp4_choice(c) && N % (32 * c.cw) == 0) return c;
    const int nsm = num_sms();
    const int nst = (K + fp4d::KS - 1) / fp4d::KS;
    const int ks_cap = nst > 8 ? 8 : nst;
    const long target = (long)(1.3 * nsm);
    const int cws[4] = {4, 8, 2, 1};
    for (int cw : cws) {
        if (N % (32 * cw)) continue;
        const long tiles = (long)(N / (32 * cw)) * mblocks;
        int ks = 1;
        while (ks < ks_cap && tiles * ks < target) ++ks;
        return {cw, ks, 0};
    }
    return c;
}

}  // namespace

// NVFP4 W4A16 with 9..16 tokens: the decode kernel (two token tiles) instead of the tensor-core
// GEMM on layers up to 32 Mi weights (5120 x 5120 at M = 9 / 12 / 16: 11.9 / 12.9 / 14.8 us
// against 16.9 / 16.9 / 17.1) and at 9 tokens on layers with K <= 8192 (17408 x 5120: 22.8
// against 36.9 us); wider or deeper layers at more tokens keep the tensor cores.
bool prefer_fp4_decode(int M, int N, int K) {
    if (M < 1 || M > 16) return false;
    if (M < kFp4PrefillMinM) return true;
    return (long long)N * K <= 32LL * 1024 * 1024 || (M <= 9 && K <= 8192);
}

namespace {

// One decode GEMM call: E stacked weight matrices, grp.n expert row groups (1 for a plain GEMM).
struct Fp4Call {
    const uint16_t *a;
    const uint8_t *w;
    const void *scale;
    const float *global_scale;  // one per expert
    void *c;
    int c_dtype, M, N, K, E, NT, rows_alloc;
    ExpertRows grp;
    unsigned int *cnt, *rowmax;
    float *part;
};

}  // namespace

template <int CW, int NT>
static int launch_fp4d_t(const Fp4Call &q, Fp4Choice ch, cudaStream_t st) {
    constexpr int BN = 32 * CW;
    const int N = q.N, K = q.K;
    const int nst = (K + fp4d::KS - 1) / fp4d::KS;
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
        int per_sm = fp4_ctas_per_sm(CW, NT, max_st, rows);
        const int fill = (int)((grid_ctas + nsm - 1) / nsm);
        if (fill < per_sm) per_sm = fill;
        const int fixed = fp4d::Lay(CW, 0, max_st, rows).total + 2048;
        const int per_stage = fp4d::Lay(CW, 1, max_st, rows).total - fp4d::Lay(CW, 0, max_st, rows).total;
        S = (kSmemPerSm / per_sm - fixed) / per_stage;
        S = S < 2 ? 2 : (S > fp4d::kMaxStages ? fp4d::kMaxStages : S);
    }
    const size_t smem = 1024 + (size_t)fp4d::Lay(CW, S, max_st, rows).total;
    if (smem > (size_t)kSmemPerCta) return -1;
    const uint64_t E = (uint64_t)q.E;
    CUtensorMap w_map, sc_map;
    if (!make_map_3d(&w_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, q.w, (uint64_t)K / 2, N, E, (uint64_t)K / 2,
                     (uint64_t)N * K / 2, fp4d::KS / 2, 32, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_3d(&sc_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, q.scale, N, K / 16, E, (uint64_t)N, (uint64_t)N * (K / 16),
                     BN, 16, CU_TENSOR_MAP_SWIZZLE_NONE))
        return -1;
    auto kern = fp4d::nvfp4_decode_kernel<CW, NT>;
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
    W4_CUDA_TRY(launch_decode(kern, grid, block, smem, st, 1u, w_map, sc_map, q.a, q.global_scale, q.c, q.c_dtype, q.M,
                              N, K, nst, max_st, S, pre, q.rows_alloc, q.grp, q.part, q.cnt, q.rowmax));
    return W4_OK;
}

template <int NT>
static int launch_fp4d_nt(const Fp4Call &q, Fp4Choice ch, cudaStream_t st) {
    switch (ch.cw) {
        case 8: return launch_fp4d_t<8, NT>(q, ch, st);
        case 4: return launch_fp4d_t<4, NT>(q, ch, st);
        case 2: return launch_fp4d_t<2, NT>(q, ch, st);
        case 1: return launch_fp4d_t<1, NT>(q, ch, st);
        default: return -1;
    }
}

// K a multiple of 64: whole 16-k scale blocks and 16-byte activation copies; a partial last stage
// reads zero codes, scales and activations.
static bool fp4_decode_shape_ok(int N, int K) { return N % 32 == 0 && K % 64 == 0; }

static int fp4_max_rows(const int *off, int n) {
    if (!off || n < 1 || n > kMaxExperts || off[0] != 0) return -1;
    int m = 0;
    for (int e = 0; e < n; ++e) {
        if (off[e + 1] < off[e]) return -1;
        m = off[e + 1] - off[e] > m ? off[e + 1] - off[e] : m;
    }
    return m;
}

static size_t fp4_split_bytes_for(const int *off, int n, int N, int K) {
    const int mr = fp4_max_rows(off, n);
    if (mr < 0 || !fp4_decode_shape_ok(N, K)) return 0;
    const int NT = mr <= 8 ? 1 : 2;
    ExpertRows g;
    if (!expert_rows(g, off, n, 8 * NT)) return 0;
    const Fp4Choice ch = fp4_choose(g.blk0[n], N, K);
    const int nst = (K + fp4d::KS - 1) / fp4d::KS;
    const int ks = ch.ks > nst ? nst : ch.ks;
    return ks > 1 ? (size_t)ks * off[n] * N * 4 : 0;
}

size_t nvfp4_decode_split_bytes(int M, int N, int K) {
    if (M < 1) return 0;
    const int off[2] = {0, M};
    return fp4_split_bytes_for(off, 1, N, K);
}

size_t nvfp4_decode_grouped_split_bytes(const int *off, int n, int N, int K) {
    return fp4_split_bytes_for(off, n, N, K);
}

static int run_fp4_decode(Fp4Call &q, const int *off, int n, int scale_dtype, void *sync, void *ws, size_t ws_bytes,
                          cudaStream_t st) {
    const char *env = std::getenv("W4_NVFP4_DECODE");
    if (env && env[0] == 'r') return -1;  // tuning override "reg": the register-streamed kernel runs
    const int mr = fp4_max_rows(off, n);
    if (mr < 0 || !fp4_decode_shape_ok(q.N, q.K)) return -1;
    // E4M3 block scales only: a bf16 scale times an e2m1 code need not be an f16
    if (scale_dtype != W4_E4M3 || !aligned(q.a, 16) || !aligned(q.w, 16) || !aligned(q.scale, 16)) return -1;
    q.NT = mr <= 8 ? 1 : 2;
    q.rows_alloc = mr < 8 * q.NT ? mr : 8 * q.NT;
    q.M = off[n];
    if (!expert_rows(q.grp, off, n, 8 * q.NT)) return -1;
    if (q.M == 0) return W4_OK;
    Fp4Choice ch = fp4_choose(q.grp.blk0[n], q.N, q.K);
    const int nst = (q.K + fp4d::KS - 1) / fp4d::KS;
    if (ch.ks > nst) ch.ks = nst;
    const long tiles = (long)(q.N / (32 * ch.cw)) * q.grp.blk0[n];
    // The K split needs the workspace: fp32 partials and one counter per tile in the sync area.
    if (ch.ks > 1 && (!sync || !ws || !aligned(ws, 16) || ws_bytes < (size_t)ch.ks * q.M * q.N * 4 ||
                      tiles > (long)kSyncTileCounters))
        ch.ks = 1;
    q.cnt = static_cast<unsigned int *>(sync);
    q.part = static_cast<float *>(ws);
    return q.NT == 1 ? launch_fp4d_nt<1>(q, ch, st) : launch_fp4d_nt<2>(q, ch, st);
}

// W4_OK / a W4 error, or -1 when the shape or tensor maps are not handled here.
int nvfp4_gemv_decode(const uint16_t *a, const uint8_t *w, const void *scale, int scale_dtype,
                      const float *global_scale, void *c, int c_dtype, int M, int N, int K, void *sync, void *ws,
                      size_t ws_bytes, unsigned int *rowmax, cudaStream_t st) {
    if (M < 1) return -1;
    Fp4Call q{};
    q.a = a, q.w = w, q.scale = scale, q.global_scale = global_scale, q.c = c, q.c_dtype = c_dtype;
    q.N = N, q.K = K, q.E = 1, q.rowmax = rowmax;
    const int off[2] = {0, M};
    return run_fp4_decode(q, off, 1, scale_dtype, sync, ws, ws_bytes, st);
}

int nvfp4_gemv_decode_grouped(const uint16_t *a, const uint8_t *w, const void *scale, int scale_dtype,
                              const float *global_scale, const int *off, int n, void *c, int c_dtype, int N, int K,
                              void *sync, void *ws, size_t ws_bytes, cudaStream_t st) {
    Fp4Call q{};
    q.a = a, q.w = w, q.scale = scale, q.global_scale = global_scale, q.c = c, q.c_dtype = c_dtype;
    q.N = N, q.K = K, q.E = n, q.rowmax = nullptr;
    return run_fp4_decode(q, off, n, scale_dtype, sync, ws, ws_bytes, st);
}

int take_fp4d_wait_status() {
    unsigned int v = 0;
    W4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_fp4d_timeout, sizeof(v)));
    if (v) {
        const unsigned int zero = 0;
        W4_CUDA_TRY(cudaMemcpyToSymbol(g_fp4d_timeout, &zero, sizeof(zero)));
        set_error("a device-side wait expired in the NVFP4 decode GEMM");
        return W4_ERR_TIMEOUT;
    }
    return W4_OK;
}

}  // namespace w4
