// gptq_prefill.cu -- GPTQ int4 W4A16 prefill GEMM on the 5th-generation tensor
// cores (tcgen05, sm_100a).
//
// Contract: the W4A16 GEMM of w4_gptq_gemm, C[m,n] = sum_k A[m,k] * w[k,n] with
// w = s[g,n] * (q[k,n] - zero[g,n]); the reference's prefill kernel is launch()
// of kernels/esimd_dpas/dpas_s4_gptq_db48.cpp:148-246 (same formula, s32
// groups there, W4A16 here per the checkpoint layout).
//
// One CTA computes a 128 x BN tile of C (BN = 256 or 128) with the fp32
// accumulator in tensor memory (TMEM, BN columns x 128 lanes).  N need only be
// a multiple of 32: the last column tile reads past N through the tensor maps'
// zero fill (zero codes, scales and zeros dequantise to 0) and stores only the
// 32-column chunks below N.  Grouped (MoE) GEMMs run the same kernel: the
// weights are E stacked matrices read through 3-D tensor maps (expert = z),
// each CTA's 128-row tile belongs to one expert (ExpertRows), and it stores
// only that expert's rows; a plain GEMM is the one-expert case.  Eighteen
// warps, specialised:
//   warp 0     TMA producer: per 64-deep k-block, the A tile (128 x 64 bf16,
//              128-byte swizzled) and the raw weight pieces (qweight 8 x BN
//              int32, the group's scale row and packed zero row) into ring
//              stage s, all completing on full[s].
//   warp 1     MMA issuer: allocates TMEM; per k-block one elected thread
//              issues four tcgen05.mma kind::f16 (M=128, N=BN, K=16) from
//              shared-memory descriptors, then tcgen05.commit frees the A/raw
//              stage (empty[s]) and the B stage (bempty[j]).
//   warps 2-17 dequantisers: TPC threads share column n; each turns 8/TPC of the
//              k-block's eight int32 words of column n into 8 bf16 (or f16)
//              weights bf16((q - z) * s) apiece, written as 16-byte chunks of row
//              n of the K-major, 128-byte-swizzled B tile, then fences the writes
//              to the async proxy and arrives on bfull[j].  Warps 2-5 then read
//              the accumulator out of TMEM (32 lanes each) and store C.
// (q - z) is exact in bf16; the product is rounded once to the MMA input type.
//
// FP4: the same GEMM for NVFP4 weights with bf16 activations (W4A16; the
// reference operator nvfp4_gemm_w4a16, kernels/nvfp4/bench_nvfp4_m1.py:58-96, at
// prefill sizes).  The raw weight pieces are the k-block's 32 code bytes of each
// of the BN columns ([N, K/2] K-contiguous) and its four E4M3 block-scale rows;
// a dequantiser turns 8 codes into e2m1 * scale in bf16 (exact: at most six
// significant bits) and the epilogue multiplies by the fp32 tensor scale.
// Every mbarrier wait is bounded (tma_util.cuh): on expiry the CTA stops its
// loops, the MMA thread still signals completion, TMEM is freed, and
// w4_check_device_status() reports W4_ERR_TIMEOUT.  No copy uses multicast.
#include <cstdio>
#include <cstdlib>
#include <type_traits>

#include <cuda_fp8.h>

#include "nvfp4_util.cuh"
#include "tma_util.cuh"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

static __device__ unsigned int g_prefill_timeout;  // a bounded wait expired (sticky until read)

namespace pf {

constexpr int BM = 128, BK = 64;
constexpr int SB = 3;         // dequantised-B ring depth
constexpr int kDeqWarps = 16;  // two threads per column of a 256-wide tile
constexpr int kThreads = (2 + kDeqWarps) * 32;

// MT: 128-row A tiles per CTA sharing one dequantised B tile (1 or 2).
template <int BN, int MT, bool FP4 = false> struct Layout {
    static constexpr int S = MT == 2 ? 3 : 4;                // A + raw-weight ring depth
    static constexpr uint32_t A_BYTES = MT * BM * BK * 2;    // 16 KB per 128 rows
    static constexpr uint32_t B_BYTES = BN * BK * 2;         // 32 KB at BN = 256
    static constexpr uint32_t QW_BYTES = (BK / 8) * BN * 4;  // 8 KB (FP4: BN x 32 code bytes, the same)
    static constexpr uint32_t SC_BYTES = FP4 ? (BK / 16) * BN : BN * 2;  // f16 scale row / 4 E4M3 rows
    static constexpr uint32_t ZR_SLOT = 128;                 // one packed zero row (BN/2 bytes), 128-aligned
    static constexpr uint32_t A_OFF = 0;
    static constexpr uint32_t B_OFF = A_OFF + S * A_BYTES;
    static constexpr uint32_t QW_OFF = B_OFF + SB * B_BYTES;
    static constexpr uint32_t SC_OFF = QW_OFF + S * QW_BYTES;
    static constexpr uint32_t ZR_OFF = SC_OFF + S * SC_BYTES;
    static constexpr uint32_t BAR_OFF = ZR_OFF + S * ZR_SLOT;  // full[S] empty[S] bfull[SB] bempty[SB] done
    static constexpr uint32_t MISC_OFF = BAR_OFF + (2 * S + 2 * SB + 1) * 8;
    static constexpr uint32_t TOTAL = MISC_OFF + 16;
    static_assert(TOTAL + 1024 <= 227 * 1024, "fits the shared memory of one CTA");
    static_assert(B_OFF % 1024 == 0 && QW_OFF % 128 == 0 && SC_OFF % 128 == 0 && ZR_OFF % 128 == 0,
                  "TMA destinations: swizzled tiles 1024-aligned, others 128-aligned");
    static_assert(BN / 2 <= ZR_SLOT, "zero row fits its slot");
};

// ---- tcgen05 helpers (cta_group::1) ----
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, both operands K-major.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the mbarrier when every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 32 lanes x 32 consecutive 32-bit TMEM columns into 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row
// groups 1024 bytes apart (SBO), version 1 (sm_100), base offset 0 (tiles are
// 1024-aligned; a K step inside the swizzle atom moves the start address).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: D f32, A/B f16 (0) or bf16 (1), both K-major, N>>3, M>>4.
template <typename T, int BN> __host__ __device__ constexpr uint32_t idesc_f16() {
    return (1u << 4) | ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 7) |
           ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 10) | ((uint32_t)(BN >> 3) << 17) |
           ((uint32_t)(BM >> 4) << 24);
}

template <typename T> struct Deq;
template <> struct Deq<__nv_bfloat16> {
    static constexpr uint32_t kMagic = 0x43004300u, kMagicHalf = 0x4300u;  // bf16 128 + q
    static __device__ __forceinline__ uint32_t scale2(uint16_t s_f16) {
        const __nv_bfloat16 b = __float2bfloat16_rn(__half2float(__ushort_as_half(s_f16)));
        const uint32_t u = __bfloat16_as_ushort(b);
        return u | (u << 16);
    }
    static __device__ __forceinline__ uint32_t sub_mul(uint32_t q, uint32_t z, uint32_t s) {
        __nv_bfloat162 d = __hsub2(*reinterpret_cast<__nv_bfloat162 *>(&q), *reinterpret_cast<__nv_bfloat162 *>(&z));
        d = __hmul2(d, *reinterpret_cast<__nv_bfloat162 *>(&s));
        return *reinterpret_cast<uint32_t *>(&d);
    }
};
template <> struct Deq<__half> {
    static constexpr uint32_t kMagic = 0x64006400u, kMagicHalf = 0x6400u;  // f16 1024 + q
    static __device__ __forceinline__ uint32_t scale2(uint16_t s_f16) { return (uint32_t)s_f16 | ((uint32_t)s_f16 << 16); }
    static __device__ __forceinline__ uint32_t sub_mul(uint32_t q, uint32_t z, uint32_t s) {
        __half2 d = __hsub2(*reinterpret_cast<__half2 *>(&q), *reinterpret_cast<__half2 *>(&z));
        d = __hmul2(d, *reinterpret_cast<__half2 *>(&s));
        return *reinterpret_cast<uint32_t *>(&d);
    }
};

// Bounded wait that also gives up at once when another role already failed.
__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    const uint32_t b = smem_u32(bar);
    if (mbar_try_wait(b, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(b, parity)) {
        if (*abort_flag) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1;
            atomicExch(&g_prefill_timeout, 1u);
            return false;
        }
    }
    return true;
}

template <typename T, int BN, int MT, bool FP4>
__global__ void __launch_bounds__(kThreads, 1)
gptq_prefill_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap qw_map,
                    const __grid_constant__ CUtensorMap sc_map, const __grid_constant__ CUtensorMap zr_map,
                    int has_z, void *__restrict__ C, int c_dtype, int M, int N, int K, int gs, int zero_offset,
                    int kb_per_split, float *__restrict__ partial, const float *__restrict__ w_global,
                    const __grid_constant__ ExpertRows grp) {
    static_assert(!FP4 || std::is_same<T, __nv_bfloat16>::value, "NVFP4 weights meet bf16 activations");
    using Lay = Layout<BN, MT, FP4>;
    constexpr int S = Lay::S;
    extern __shared__ uint8_t smem_dyn[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + Lay::BAR_OFF);
    uint64_t *empty = full + S;
    uint64_t *bfull = empty + S;
    uint64_t *bempty = bfull + SB;
    uint64_t *done = bempty + SB;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + Lay::MISC_OFF);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + Lay::MISC_OFF + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // this CTA's rows: tile blockIdx.x - blk0[ex] of expert ex, rows [m0, m_end) stored
    const int ex = expert_of_block(grp, blockIdx.x);
    const int m0 = grp.row0[ex] + ((int)blockIdx.x - grp.blk0[ex]) * BM * MT, m_end = grp.row0[ex + 1];
    const int n0 = blockIdx.y * BN;
    // split-K: this CTA reduces k-blocks [kb0, kb0 + nk) and, when split, writes an
    // fp32 partial tile that a second kernel sums
    const int kb0 = blockIdx.z * kb_per_split;
    const int nk = min(kb_per_split, K / BK - kb0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int j = 0; j < SB; ++j) {
            mbar_init(&bfull[j], kDeqWarps);
            mbar_init(&bempty[j], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, MT * BN);  // one accumulator per 128-row A tile
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            // A: the whole BM * MT-row tile (rows of the next expert or past M included: they meet
            // only accumulator rows that are never stored).  Loading only the 32-row boxes that
            // hold this tile's rows measured 12 % slower on the MoE shapes.
            const uint32_t tx = Lay::A_BYTES + Lay::QW_BYTES + Lay::SC_BYTES + (has_z ? BN / 2 : 0);
            for (int i = 0; i < nk; ++i) {
                const int s = i % S;
                if (i >= S && !pf_wait(&empty[s], (uint32_t)(((i / S) - 1) & 1), abort_flag)) break;
                const int kb = kb0 + i;
                const int g = (kb * BK) / gs;
                mbar_arrive_expect_tx(&full[s], tx);
                tma_load_2d(sm + Lay::A_OFF + s * Lay::A_BYTES, &a_map, kb * BK, m0, &full[s]);
                if constexpr (FP4) {
                    tma_load_3d(sm + Lay::QW_OFF + s * Lay::QW_BYTES, &qw_map, kb * (BK / 2), n0, ex, &full[s]);
                    tma_load_3d(sm + Lay::SC_OFF + s * Lay::SC_BYTES, &sc_map, n0, kb * (BK / 16), ex, &full[s]);
                } else {
                    tma_load_3d(sm + Lay::QW_OFF + s * Lay::QW_BYTES, &qw_map, n0, kb * (BK / 8), ex, &full[s]);
                    tma_load_3d(sm + Lay::SC_OFF + s * Lay::SC_BYTES, &sc_map, n0, g, ex, &full[s]);
                    if (has_z) tma_load_3d(sm + Lay::ZR_OFF + s * Lay::ZR_SLOT, &zr_map, n0 / 8, g, ex, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16<T, BN>();
            for (int i = 0; i < nk; ++i) {
                const int s = i % S, j = i % SB;
                if (!pf_wait(&full[s], (uint32_t)((i / S) & 1), abort_flag)) break;
                if (!pf_wait(&bfull[j], (uint32_t)((i / SB) & 1), abort_flag)) break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sm + Lay::A_OFF + s * Lay::A_BYTES);
                const uint32_t b_addr = smem_u32(sm + Lay::B_OFF + j * Lay::B_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
#pragma unroll
                    for (int mh = 0; mh < MT; ++mh)  // same B tile, A rows 128 * mh .. +127
                        mma_f16_ss(tmem + (uint32_t)(mh * BN), sw128_kmajor_desc(a_addr + mh * (BM * 128) + kk * 32),
                                   sw128_kmajor_desc(b_addr + kk * 32), idesc, (i | kk) != 0);
                tc_commit(&empty[s]);
                tc_commit(&bempty[j]);
            }
            tc_commit(done);  // also on failure: nothing in flight, the epilogue still ends
        }
    } else {
        // ---------------- dequantisers ----------------
        constexpr int TPC = kDeqWarps * 32 / BN;  // threads per column
        const int dt = threadIdx.x - 64;
        const int n = dt % BN, r0 = dt / BN;
        const uint32_t zsh = 4 * (n & 7);
        const uint32_t zbase = Deq<T>::kMagicHalf + (has_z ? (uint32_t)zero_offset : 8u);
        for (int i = 0; i < nk; ++i) {
            const int s = i % S, j = i % SB;
            bool ok = pf_wait(&full[s], (uint32_t)((i / S) & 1), abort_flag);
            if (ok && i >= SB) ok = pf_wait(&bempty[j], (uint32_t)(((i / SB) - 1) & 1), abort_flag);
            if (!__all_sync(0xffffffffu, ok)) break;
            if constexpr (FP4) {
                // thread r0 of column n dequantises code chunks [r0 * CPT, (r0 + 1) * CPT) of the
                // k-block (a chunk = 8 k = 4 code bytes; 16-k block scale row = chunk / 2)
                constexpr int CPT = 8 / TPC;
                const uint8_t *codes = sm + Lay::QW_OFF + s * Lay::QW_BYTES + n * (BK / 2) + r0 * CPT * 4;
                const uint8_t *srow = sm + Lay::SC_OFF + s * Lay::SC_BYTES + n;
                uint8_t *brow = sm + Lay::B_OFF + j * Lay::B_BYTES + n * 128;
                uint32_t cw[CPT];
                if constexpr (CPT == 4) {
                    const uint4 u = *reinterpret_cast<const uint4 *>(codes);
                    cw[0] = u.x, cw[1] = u.y, cw[2] = u.z, cw[3] = u.w;
                } else {
#pragma unroll
                    for (int t = 0; t < CPT; ++t) cw[t] = reinterpret_cast<const uint32_t *>(codes)[t];
                }
#pragma unroll
                for (int t = 0; t < CPT; ++t) {
                    const int kr = r0 * CPT + t;
                    const __half_raw sh = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)srow[(kr >> 1) * BN], __NV_E4M3);
                    const uint32_t sb = __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(__ushort_as_half(sh.x))));
                    const uint32_t sc2 = sb | (sb << 16);
                    uint32_t v01, v23, v45, v67;
                    e2m1x4_to_bf16(cw[t], v01, v23);
                    e2m1x4_to_bf16(cw[t] >> 16, v45, v67);
                    uint4 o;  // k0..k7 in order
                    o.x = bf16x2_mul(v01, sc2);
                    o.y = bf16x2_mul(v23, sc2);
                    o.z = bf16x2_mul(v45, sc2);
                    o.w = bf16x2_mul(v67, sc2);
                    *reinterpret_cast<uint4 *>(brow + ((kr ^ (n & 7)) << 4)) = o;
                }
                fence_proxy_async();  // make the generic-proxy writes visible to the tensor core
                __syncwarp();
                if (lane == 0) mbar_arrive(&bfull[j]);
                continue;
            }
            const uint16_t sbits = reinterpret_cast<const uint16_t *>(sm + Lay::SC_OFF + s * Lay::SC_BYTES)[n];
            const uint32_t zq =
                has_z ? (reinterpret_cast<const uint32_t *>(sm + Lay::ZR_OFF + s * Lay::ZR_SLOT)[n >> 3] >> zsh) & 15u
                      : 0u;
            const uint32_t zc = (zbase + zq) * 0x00010001u;
            const uint32_t sc = Deq<T>::scale2(sbits);
            const uint32_t *qw = reinterpret_cast<const uint32_t *>(sm + Lay::QW_OFF + s * Lay::QW_BYTES);
            uint8_t *brow = sm + Lay::B_OFF + j * Lay::B_BYTES + n * 128;
#pragma unroll
            for (int t = 0; t < 8 / TPC; ++t) {  // compile-time trip count: the words interleave
                const int kr = r0 + t * TPC;
                const uint32_t w = qw[kr * BN + n];
                const uint32_t d0 = Deq<T>::sub_mul(lop3_and_or(w, 0x000F000Fu, Deq<T>::kMagic), zc, sc);
                const uint32_t d1 = Deq<T>::sub_mul(lop3_and_or(w >> 4, 0x000F000Fu, Deq<T>::kMagic), zc, sc);
                const uint32_t d2 = Deq<T>::sub_mul(lop3_and_or(w >> 8, 0x000F000Fu, Deq<T>::kMagic), zc, sc);
                const uint32_t d3 = Deq<T>::sub_mul(lop3_and_or(w >> 12, 0x000F000Fu, Deq<T>::kMagic), zc, sc);
                uint4 o;  // k0..k7 in order: d_q holds (k_q, k_q+4)
                o.x = __byte_perm(d0, d1, 0x5410);
                o.y = __byte_perm(d2, d3, 0x5410);
                o.z = __byte_perm(d0, d1, 0x7632);
                o.w = __byte_perm(d2, d3, 0x7632);
                *reinterpret_cast<uint4 *>(brow + ((kr ^ (n & 7)) << 4)) = o;
            }
            fence_proxy_async();  // make the generic-proxy writes visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&bfull[j]);
        }
        // ---------------- epilogue (warps 2-5: TMEM lanes 32*(warp%4) ...) ----------------
        if (warp < 6) {
            const bool ok = pf_wait(done, 0u, abort_flag);
            (void)ok;
            tc_fence_after();
            const int q = warp & 3;
            const float gsc = w_global ? w_global[ex] : 1.0f;  // NVFP4 tensor scale of this expert
#pragma unroll 1
            for (int cc = 0; cc < MT * BN; cc += 32) {
                const int mh = cc / BN, c0 = cc % BN;
                const int row = m0 + mh * BM + 32 * q + lane;
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)cc, v);
                if (w_global) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * gsc);
                }
                if (row < m_end && n0 + c0 < N) {  // N % 32 == 0: a chunk is wholly inside or outside
                    const size_t base = (size_t)row * N + n0 + c0;
                    if (partial) {
                        float4 *dst = reinterpret_cast<float4 *>(partial + (size_t)blockIdx.z * M * N + base);
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            dst[e] = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                                 __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
                    } else if (c_dtype == W4_F32) {
                        float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(C) + base);
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            dst[e] = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                                 __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
                    } else {
                        uint32_t p[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const float x0 = __uint_as_float(v[2 * e]), x1 = __uint_as_float(v[2 * e + 1]);
                            if (c_dtype == W4_BF16) {
                                __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
                                p[e] = *reinterpret_cast<uint32_t *>(&h);
                            } else {
                                __half2 h = __floats2half2_rn(x0, x1);
                                p[e] = *reinterpret_cast<uint32_t *>(&h);
                            }
                        }
                        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(C) + base);
#pragma unroll
                        for (int e = 0; e < 4; ++e) dst[e] = make_uint4(p[4 * e], p[4 * e + 1], p[4 * e + 2], p[4 * e + 3]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, MT * BN);
    }
}

// Sum of the split-K partial tiles, converted to the output type.
__global__ void splitk_reduce_kernel(const float *__restrict__ partial, int splits, long mn, void *__restrict__ C,
                                     int c_dtype) {
    const long i4 = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i4 >= mn) return;
    float4 acc = *reinterpret_cast<const float4 *>(partial + i4);
    for (int sp = 1; sp < splits; ++sp) {
        const float4 v = *reinterpret_cast<const float4 *>(partial + (size_t)sp * mn + i4);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    if (c_dtype == W4_F32) {
        *reinterpret_cast<float4 *>(static_cast<float *>(C) + i4) = acc;
    } else if (c_dtype == W4_BF16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
        *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(C) + i4) =
            make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
    } else {
        __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
        *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(C) + i4) =
            make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
    }
}

// Shared memory of one prefill kernel instantiation (the template argument), opted in once per
// device.
template <auto kern>
static int prepare(size_t smem) {
    static std::mutex mu;
    static bool set_dev[128] = {};
    int dev = 0;
    W4_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 128 && !set_dev[dev]) {
        W4_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        set_dev[dev] = true;
    }
    return W4_OK;
}

// GPTQ weights: E stacked [K/8, N] qweight, [K/gs, N] scales, [K/gs, N/8] qzeros (or none).
template <typename T, int BN, int MT>
static int launch(const void *a, const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales, void *c,
                  int c_dtype, const ExpertRows &g, int E, int M, int N, int K, int gs, int zero_offset, int ksplit,
                  float *partial, cudaStream_t st) {
    using Lay = Layout<BN, MT>;
    const CUtensorMapDataType adt =
        std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint64_t ng = (uint64_t)(K / gs);
    CUtensorMap a_map, qw_map, sc_map, zr_map;
    if (!make_map_2d(&a_map, adt, a, K, M, (uint64_t)K * 2, BK, BM * MT, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_3d(&qw_map, CU_TENSOR_MAP_DATA_TYPE_INT32, qweight, N, K / 8, E, (uint64_t)N * 4,
                     (uint64_t)(K / 8) * N * 4, BN, BK / 8, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_3d(&sc_map, CU_TENSOR_MAP_DATA_TYPE_UINT16, scales, N, ng, E, (uint64_t)N * 2, ng * N * 2, BN, 1,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return -1;
    const int has_z = qzeros != nullptr;
    if (has_z) {
        if (!make_map_3d(&zr_map, CU_TENSOR_MAP_DATA_TYPE_INT32, qzeros, N / 8, ng, E, (uint64_t)N / 2, ng * N / 2,
                         BN / 8, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
            return -1;
    } else {
        zr_map = sc_map;  // unused
    }
    constexpr auto kern = gptq_prefill_kernel<T, BN, MT, false>;
    const size_t smem = Lay::TOTAL + 1024;
    if (const int rc = prepare<kern>(smem)) return rc;
    const int nk = K / BK;
    const int kb_per_split = (nk + ksplit - 1) / ksplit;
    ksplit = (nk + kb_per_split - 1) / kb_per_split;  // every split gets at least one k-block
    dim3 grid((unsigned)g.blk0[g.n], (unsigned)((N + BN - 1) / BN), (unsigned)ksplit), block(kThreads);
    kern<<<grid, block, smem, st>>>(a_map, qw_map, sc_map, zr_map, has_z, c, c_dtype, M, N, K, gs, zero_offset,
                                    kb_per_split, ksplit > 1 ? partial : nullptr, nullptr, g);
    W4_LAUNCH_CHECK();
    if (ksplit > 1) {
        const long mn = (long)M * N;  // N % 32 == 0: whole float4 groups
        splitk_reduce_kernel<<<(unsigned)((mn / 4 + 255) / 256), 256, 0, st>>>(partial, ksplit, mn, c, c_dtype);
        W4_LAUNCH_CHECK();
    }
    return W4_OK;
}

// NVFP4 weights: E stacked codes [N, K/2] (K-contiguous), E4M3 block scales [K/16, N] and one
// fp32 tensor scale per expert, with bf16 activations.
template <int BN, int MT>
static int launch_fp4(const uint16_t *a, const uint8_t *w_nk, const uint8_t *scale, const float *w_global, void *c,
                      int c_dtype, const ExpertRows &g, int E, int M, int N, int K, int ksplit, float *partial,
                      cudaStream_t st) {
    using Lay = Layout<BN, MT, true>;
    CUtensorMap a_map, qw_map, sc_map;
    if (!make_map_2d(&a_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a, K, M, (uint64_t)K * 2, BK, BM * MT,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_3d(&qw_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_nk, (uint64_t)K / 2, N, E, (uint64_t)K / 2,
                     (uint64_t)N * (K / 2), BK / 2, BN, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_3d(&sc_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, scale, N, K / 16, E, (uint64_t)N, (uint64_t)(K / 16) * N,
                     BN, BK / 16, CU_TENSOR_MAP_SWIZZLE_NONE))
        return -1;
    constexpr auto kern = gptq_prefill_kernel<__nv_bfloat16, BN, MT, true>;
    const size_t smem = Lay::TOTAL + 1024;
    if (const int rc = prepare<kern>(smem)) return rc;
    const int nk = K / BK;
    const int kb_per_split = (nk + ksplit - 1) / ksplit;
    ksplit = (nk + kb_per_split - 1) / kb_per_split;
    dim3 grid((unsigned)g.blk0[g.n], (unsigned)((N + BN - 1) / BN), (unsigned)ksplit), block(kThreads);
    kern<<<grid, block, smem, st>>>(a_map, qw_map, sc_map, sc_map, 0, c, c_dtype, M, N, K, BK, 0, kb_per_split,
                                    ksplit > 1 ? partial : nullptr, w_global, g);
    W4_LAUNCH_CHECK();
    if (ksplit > 1) {
        const long mn = (long)M * N;  // N % 32 == 0: whole float4 groups
        splitk_reduce_kernel<<<(unsigned)((mn / 4 + 255) / 256), 256, 0, st>>>(partial, ksplit, mn, c, c_dtype);
        W4_LAUNCH_CHECK();
    }
    return W4_OK;
}

}  // namespace pf

namespace pf {
static bool handled(int N, int K, int gs, int c_dtype) {
    return N > 0 && K > 0 && K % BK == 0 && gs % BK == 0 && N % 32 == 0 && c_dtype != W4_E4M3;
}

// Tiling of one call: A tiles per CTA (two 128-row tiles share each dequantised B tile once an
// expert has more than 128 rows), 256- or 128-wide column tiles, and the K split.
struct Plan {
    int mt, ks;
    bool wide;
    double cost;  // the model's estimate (us)
    ExpertRows g;
};

// Tile width and K split from a cost model in microseconds: per wave of CTAs (one per SM), the
// k-blocks of a CTA x the k-block time of the width (about 1 us at 256 columns; at 128 columns
// 0.6 of that with one A tile per CTA, where the dequantising warps' fixed cost per k-block
// dominates, and 0.8 with two, where the MMAs weigh more) plus 3 for a CTA's prologue, pipeline
// fill and epilogue; a K split adds 1 plus its fp32 partials written and read back at an
// effective 2.5 TB/s (the separate sum launch included); K is split only when the unsplit tiles fill at most half the SMs (at larger grids the
// partials cost more than the model's estimate).  Measured against the earlier fill-the-wave rule: NVFP4 5120 x 5120 M = 16, 17 us (21);
// GPTQ 5120 x 17408 M = 32, 35 us (45); 17408 x 5120 M = 256, 64 us (80); 7 experts of 17..40
// rows, 2688 x 1856, 21 us (25); unchanged choices at 5120 x 5120 M = 128..8192 and 5120 x 27648
// M = 2048.  K splits keep at least four k-blocks each, at most 8.
// false: more experts than the table holds.
static bool plan_for(const int *off, int n, int N, int K, Plan &p) {
    int max_rows = 0;
    for (int e = 0; e < n; ++e) max_rows = off[e + 1] - off[e] > max_rows ? off[e + 1] - off[e] : max_rows;
    p.mt = max_rows > BM ? 2 : 1;
    if (!expert_rows(p.g, off, n, BM * p.mt)) return false;
    const long nsm = num_sms(), blocks = p.g.blk0[n], nk = K / BK;
    const double partial_us_per_split = (double)off[n] * N * 8 / 2.5e6;  // fp32 written + read
    long ks_max = nk / 4;
    if (ks_max > 8) ks_max = 8;
    if (ks_max < 1) ks_max = 1;
    double best = 0;
    p.wide = false;
    p.ks = 1;
    p.cost = 0;
    for (int w = 1; w >= 0; --w) {  // 256-wide first: it wins ties
        if (w && N < 256) continue;
        const long tiles = blocks * (w ? (N + 255) / 256 : (N + 127) / 128);
        const long ks_top = 2 * tiles <= nsm ? ks_max : 1;  // split only grids that fill at most half the SMs
        for (long ks = 1; ks <= ks_top; ++ks) {
            const double waves = (double)((tiles * ks + nsm - 1) / nsm);
            const double kb = (double)((nk + ks - 1) / ks);
            const double t =
                waves * (kb * (w ? 1.0 : (p.mt == 2 ? 0.8 : 0.6)) + 3.0) + (ks > 1 ? 1.0 + partial_us_per_split * ks : 0.0);
            if (best == 0 || t < best - 1e-9) {
                best = t;
                p.wide = w == 1;
                p.ks = (int)ks;
                p.cost = t;
            }
        }
    }
    // tuning override W4_PREFILL="wide,ks" (wide 1: 256-column tiles, 0: 128; ks 1..8)
    if (const char *e = std::getenv("W4_PREFILL")) {
        int w = -1, k = 0;
        if (std::sscanf(e, "%d,%d", &w, &k) == 2 && (w == 0 || (w == 1 && N >= 256)) && k >= 1 && k <= 8 &&
            k <= K / BK) {
            p.wide = w == 1;
            p.ks = k;
        }
    }
    return true;
}

static size_t split_bytes_of(const int *off, int n, int N, int K) {
    Plan p;
    if (!plan_for(off, n, N, K, p) || p.ks <= 1) return 0;
    return (size_t)p.ks * off[n] * N * sizeof(float);
}

// A plain call whose tiles leave the last wave partly empty (5120^2 at M = 2048: 160 tiles of
// 256 x 256 for 148 SMs) runs as two calls along M: the row blocks that fill whole waves
// unsplit, the rest as a second call that the plan may split along K.  Returns the rows of the
// first part when the model predicts the pair faster (2 us allowed for the second launch),
// else 0.
static int tail_rows(int M, int N, int K) {
    if (std::getenv("W4_PREFILL")) return 0;  // a forced plan applies to the whole call
    const int off[2] = {0, M};
    Plan whole;
    if (!plan_for(off, 1, N, K, whole)) return 0;
    const long nsm = num_sms();
    const long ntile = whole.wide ? (N + 255) / 256 : (N + 127) / 128;
    const long tiles = (long)whole.g.blk0[1] * ntile;
    const long full_waves = tiles / nsm;
    if (full_waves == 0 || tiles % nsm == 0) return 0;
    const int M1 = (int)(full_waves * nsm / ntile) * BM * whole.mt;
    if (M1 <= 0 || M1 >= M) return 0;
    const int off1[2] = {0, M1}, off2[2] = {0, M - M1};
    Plan p1, p2;
    if (!plan_for(off1, 1, N, K, p1) || !plan_for(off2, 1, N, K, p2)) return 0;
    return p1.cost + p2.cost + 2.0 < whole.cost ? M1 : 0;
}

static size_t split_bytes(const int *off, int n, int N, int K) {
    if (n == 1) {
        if (const int M1 = tail_rows(off[1], N, K)) {
            const int off1[2] = {0, M1}, off2[2] = {0, off[1] - M1};
            const size_t b1 = split_bytes_of(off1, 1, N, K), b2 = split_bytes_of(off2, 1, N, K);
            return b1 > b2 ? b1 : b2;
        }
    }
    return split_bytes_of(off, n, N, K);
}

static int gptq_run(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                    const uint16_t *scales, const int *off, int n, int E, void *c, int c_dtype, int N, int K, int gs,
                    int zero_offset, void *split_ws, size_t split_ws_bytes, cudaStream_t st, bool tail = true) {
    if (!handled(N, K, gs, c_dtype)) return -1;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(qweight) |
         reinterpret_cast<uintptr_t>(scales) | reinterpret_cast<uintptr_t>(qzeros)) & 15)
        return -1;
    if (tail && n == 1) {
        if (const int M1 = tail_rows(off[1], N, K)) {
            const int off1[2] = {0, M1}, off2[2] = {0, off[1] - M1};
            const size_t csz = c_dtype == W4_F32 ? 4 : 2;
            int rc = gptq_run(a, a_dtype, qweight, qzeros, scales, off1, 1, 1, c, c_dtype, N, K, gs, zero_offset,
                              split_ws, split_ws_bytes, st, false);
            if (rc) return rc;
            return gptq_run(static_cast<const uint16_t *>(a) + (size_t)M1 * K, a_dtype, qweight, qzeros, scales, off2,
                            1, 1, static_cast<char *>(c) + (size_t)M1 * N * csz, c_dtype, N, K, gs, zero_offset,
                            split_ws, split_ws_bytes, st, false);
        }
    }
    Plan p;
    if (!plan_for(off, n, N, K, p)) return -1;
    const int M = off[n];
    if (M == 0) return W4_OK;
    int ks = p.ks;
    if (ks > 1 && (!split_ws || split_ws_bytes < (size_t)ks * M * N * sizeof(float))) ks = 1;
    float *partial = static_cast<float *>(split_ws);
#define W4_PF_LAUNCH(TT, BNV, MTV) \
    launch<TT, BNV, MTV>(a, qweight, qzeros, scales, c, c_dtype, p.g, E, M, N, K, gs, zero_offset, ks, partial, st)
    if (a_dtype == W4_BF16) {
        if (p.mt == 2) return p.wide ? W4_PF_LAUNCH(__nv_bfloat16, 256, 2) : W4_PF_LAUNCH(__nv_bfloat16, 128, 2);
        return p.wide ? W4_PF_LAUNCH(__nv_bfloat16, 256, 1) : W4_PF_LAUNCH(__nv_bfloat16, 128, 1);
    }
    if (p.mt == 2) return p.wide ? W4_PF_LAUNCH(__half, 256, 2) : W4_PF_LAUNCH(__half, 128, 2);
    return p.wide ? W4_PF_LAUNCH(__half, 256, 1) : W4_PF_LAUNCH(__half, 128, 1);
#undef W4_PF_LAUNCH
}

static int fp4_run(const uint16_t *a, const uint8_t *w_nk, const uint8_t *scale, const float *w_global,
                   const int *off, int n, int E, void *c, int c_dtype, int N, int K, void *split_ws,
                   size_t split_ws_bytes, cudaStream_t st, bool tail = true) {
    if (!handled(N, K, BK, c_dtype)) return -1;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w_nk) | reinterpret_cast<uintptr_t>(scale)) &
        15)
        return -1;
    if (tail && n == 1) {
        if (const int M1 = tail_rows(off[1], N, K)) {
            const int off1[2] = {0, M1}, off2[2] = {0, off[1] - M1};
            const size_t csz = c_dtype == W4_F32 ? 4 : 2;
            int rc = fp4_run(a, w_nk, scale, w_global, off1, 1, 1, c, c_dtype, N, K, split_ws, split_ws_bytes, st,
                             false);
            if (rc) return rc;
            return fp4_run(a + (size_t)M1 * K, w_nk, scale, w_global, off2, 1, 1,
                           static_cast<char *>(c) + (size_t)M1 * N * csz, c_dtype, N, K, split_ws, split_ws_bytes, st,
                           false);
        }
    }
    Plan p;
    if (!plan_for(off, n, N, K, p)) return -1;
    const int M = off[n];
    if (M == 0) return W4_OK;
    int ks = p.ks;
    if (ks > 1 && (!split_ws || split_ws_bytes < (size_t)ks * M * N * sizeof(float))) ks = 1;
    float *partial = static_cast<float *>(split_ws);
    if (p.mt == 2)
        return p.wide ? launch_fp4<256, 2>(a, w_nk, scale, w_global, c, c_dtype, p.g, E, M, N, K, ks, partial, st)
                      : launch_fp4<128, 2>(a, w_nk, scale, w_global, c, c_dtype, p.g, E, M, N, K, ks, partial, st);
    return p.wide ? launch_fp4<256, 1>(a, w_nk, scale, w_global, c, c_dtype, p.g, E, M, N, K, ks, partial, st)
                  : launch_fp4<128, 1>(a, w_nk, scale, w_global, c, c_dtype, p.g, E, M, N, K, ks, partial, st);
}
}  // namespace pf

size_t gptq_prefill_split_bytes(int M, int N, int K, int gs, int c_dtype) {
    if (M < kPrefillMinM || !pf::handled(N, K, gs, c_dtype)) return 0;
    const int off[2] = {0, M};
    return pf::split_bytes(off, 1, N, K);
}

// W4_OK / a W4 error, or -1 when this shape is not handled here (the caller
// then runs the decode kernels).  split_ws (gptq_prefill_split_bytes) holds the
// split-K partials; without it the GEMM runs unsplit.
int gptq_prefill(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                 void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset, void *split_ws,
                 size_t split_ws_bytes, cudaStream_t st) {
    const int off[2] = {0, M};
    return pf::gptq_run(a, a_dtype, qweight, qzeros, scales, off, 1, 1, c, c_dtype, N, K, gs, zero_offset, split_ws,
                        split_ws_bytes, st);
}

size_t gptq_prefill_grouped_split_bytes(const int *off, int n, int N, int K, int gs, int c_dtype) {
    if (!pf::handled(N, K, gs, c_dtype)) return 0;
    return pf::split_bytes(off, n, N, K);
}

int gptq_prefill_grouped(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                         const uint16_t *scales, const int *off, int n, void *c, int c_dtype, int N, int K, int gs,
                         int zero_offset, void *split_ws, size_t split_ws_bytes, cudaStream_t st) {
    return pf::gptq_run(a, a_dtype, qweight, qzeros, scales, off, n, n, c, c_dtype, N, K, gs, zero_offset, split_ws,
                        split_ws_bytes, st);
}

int splitk_reduce(const float *partial, int splits, long mn, void *c, int c_dtype, cudaStream_t st) {
    pf::splitk_reduce_kernel<<<(unsigned)((mn / 4 + 255) / 256), 256, 0, st>>>(partial, splits, mn, c, c_dtype);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

size_t nvfp4_w4a16_prefill_split_bytes(int M, int N, int K, int c_dtype) {
    if (prefer_fp4_decode(M, N, K) || !pf::handled(N, K, pf::BK, c_dtype)) return 0;
    const int off[2] = {0, M};
    return pf::split_bytes(off, 1, N, K);
}

// NVFP4 W4A16 on the tensor cores (M >= kFp4PrefillMinM): W4_OK / a W4 error, or -1
// when the shape is not handled here (the caller then runs the decode kernel).
int nvfp4_w4a16_prefill(const uint16_t *a, const uint8_t *w_nk, const uint8_t *scale, const float *w_global,
                        void *c, int c_dtype, int M, int N, int K, void *split_ws, size_t split_ws_bytes,
                        cudaStream_t st) {
    if (prefer_fp4_decode(M, N, K)) return -1;  // the caller runs the decode kernel
    const int off[2] = {0, M};
    return pf::fp4_run(a, w_nk, scale, w_global, off, 1, 1, c, c_dtype, N, K, split_ws, split_ws_bytes, st);
}

size_t nvfp4_w4a16_prefill_grouped_split_bytes(const int *off, int n, int N, int K, int c_dtype) {
    if (!pf::handled(N, K, pf::BK, c_dtype)) return 0;
    return pf::split_bytes(off, n, N, K);
}

int nvfp4_w4a16_prefill_grouped(const uint16_t *a, const uint8_t *w_nk, const uint8_t *scale, const float *w_global,
                                const int *off, int n, void *c, int c_dtype, int N, int K, void *split_ws,
                                size_t split_ws_bytes, cudaStream_t st) {
    return pf::fp4_run(a, w_nk, scale, w_global, off, n, n, c, c_dtype, N, K, split_ws, split_ws_bytes, st);
}

int take_prefill_wait_status() {
    unsigned int v = 0;
    W4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_prefill_timeout, sizeof(v)));
    if (v) {
        const unsigned int zero = 0;
        W4_CUDA_TRY(cudaMemcpyToSymbol(g_prefill_timeout, &zero, sizeof(zero)));
        set_error("a device-side wait expired in the GPTQ prefill GEMM");
        return W4_ERR_TIMEOUT;
    }
    return W4_OK;
}

}  // namespace w4
