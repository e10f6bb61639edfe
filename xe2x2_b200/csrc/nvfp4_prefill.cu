// nvfp4_prefill.cu -- NVFP4 x NVFP4 block-scaled GEMM on the 5th-generation
// tensor cores (tcgen05.mma kind::mxf4nvf4, sm_100a).
//
// Contract: w4_nvfp4_gemm with act_mode W4_ACT_NVFP4.  The activations are
// quantised per 16-block exactly as w4_nvfp4_quant_act does (sf_a = e4m3(amax /
// (6 a_global)), code = e2m1(a / (sf_a a_global))), then
//   C[m,n] = a_global * w_global * sum_k (e2m1_a * sf_a)[m,k] * (e2m1_w * sf_w)[n,k]
// with the fp32 sum taken by the tensor core from the block-scaled operands
// (the MMA applies one UE4M3 scale per 16 elements of each operand).  The
// reference's NVFP4 GEMM is the external operator of
// kernels/nvfp4/bench_nvfp4_m1.py:67,88 (oneDNN), W4A16 only; its LUT kernel
// (kernels/nvfp4/nibble_lut_sc.cpp:198-290) quantises activations to s8.
//
// Operands:
//   A codes  u8 [M, K/2]  (2 E2M1 per byte, low nibble = even k), TMA box
//            128 rows x 128 bytes (256 k), 128-byte swizzle, K-major.
//   W codes  u8 [N, K/2]  same.
//   scales   UE4M3, rearranged once per call into 512-byte atoms of 128 rows x
//            4 blocks (64 k): byte (r % 32) * 16 + (r / 32 % 4) * 4 + (kb % 4),
//            atoms ordered [row tile][k / 64], so a stage's four atoms are one
//            2 KB bulk copy.  tcgen05.cp (32x128b, replicated to the four lane
//            quarters) moves an atom into 4 TMEM columns for the MMA.
// Tile 128 x 128 per CTA, 256 k per pipeline stage (four K=64 MMAs).  Warp 0
// produces (TMA + bulk copies), warp 1 allocates TMEM and issues the scale
// copies and MMAs, warps 2-5 read the fp32 accumulator out of TMEM, apply the
// tensor scales and store C.  The persistent form (large grids) gives the scale
// copies a warp of their own.  Every wait is bounded; no copy uses multicast.
#include <mutex>

#include "tma_util.cuh"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

static __device__ unsigned int g_fp4pf_timeout;  // a bounded wait expired (sticky until read)

static inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---- scale rearrangement: [rows][K/16] (row stride rs, block stride ks) -> atoms ----
__global__ void nvfp4_sf_atoms_kernel(const uint8_t *__restrict__ src, int rows, int nkb, long rs, long ks,
                                      int rows_pad, uint8_t *__restrict__ dst) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const long total = (long)rows_pad * nkb;
    if (i >= total) return;
    // i enumerates destination bytes in order
    const long atom = i >> 9;
    const int within = (int)(i & 511);
    const int kchunks = nkb / 4;
    const int tile = (int)(atom / kchunks), kc = (int)(atom % kchunks);
    const int r = tile * 128 + (within >> 4) + 32 * ((within >> 2) & 3);
    const int kb = kc * 4 + (within & 3);
    dst[i] = r < rows ? src[r * rs + (long)kb * ks] : (uint8_t)0;
}

int nvfp4_sf_atoms(const uint8_t *src, int rows, int nkb, long rs, long ks, uint8_t *dst, cudaStream_t st) {
    const int rows_pad = (rows + 127) / 128 * 128;
    const long total = (long)rows_pad * nkb;
    nvfp4_sf_atoms_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, rows, nkb, rs, ks, rows_pad, dst);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

namespace fp4pf {

constexpr int BM = 128, BK = 256;  // BK in elements (128 bytes of codes)
constexpr int kThreads = 6 * 32;
constexpr uint32_t SF_ATOM = 512;

// Shared memory and TMEM plan for a 128 x BN tile.
template <int BN> struct Cfg {
    static constexpr int S = BN == 256 ? 4 : 5;                  // pipeline stages
    static constexpr int NH = BN / 128;                          // 128-row halves of the W tile
    static constexpr uint32_t A_BYTES = BM * BK / 2, B_BYTES = BN * BK / 2;
    static constexpr uint32_t SFA_BYTES = 4 * SF_ATOM, SFB_BYTES = NH * 4 * SF_ATOM;
    static constexpr uint32_t A_OFF = 0, B_OFF = A_OFF + S * A_BYTES, SFA_OFF = B_OFF + S * B_BYTES,
                              SFB_OFF = SFA_OFF + S * SFA_BYTES, BAR_OFF = SFB_OFF + S * SFB_BYTES,
                              MISC_OFF = BAR_OFF + (2 * S + 1) * 8, SMEM = MISC_OFF + 16;
    // TMEM: accumulator columns [0, BN); stage s scales at BN + s * SF_COLS (A: 16, then B: 16 NH).
    static constexpr uint32_t SF_COLS = 16 + 16 * NH, TMEM_COLS = 512;
    static_assert(BN + S * SF_COLS <= TMEM_COLS, "TMEM plan");
    // Instruction descriptor, block-scaled kind::mxf4nvf4: A/B E2M1 (1), K-major,
    // N>>3 at bit 17, scale format UE4M3 (bit 23 = 0), M>>4 at bit 24, scale ids 0.
    static constexpr uint32_t IDESC = (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
};

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 512-byte scale atom (32 rows x 16 bytes) -> TMEM lanes 0-31, 4 columns, replicated to all four lane quarters.
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void mma_fp4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                        uint32_t sfb, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %6, 0;\n"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%4], [%5], p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(sfa), "r"(sfb), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
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

// K-major operand tile, 128-byte swizzle, 8-row groups 1024 bytes apart, version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Scale atom: 32 rows of 16 bytes, no swizzle, 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t sf_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(128 >> 4) << 32) |
           ((uint64_t)1 << 46);
}

__device__ __forceinline__ bool wait_pf(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    const uint32_t b = smem_u32(bar);
    if (mbar_try_wait(b, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(b, parity)) {
        if (*abort_flag) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1;
            atomicExch(&g_fp4pf_timeout, 1u);
            return false;
        }
    }
    return true;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
nvfp4_prefill_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap w_map,
                     const uint8_t *__restrict__ sfa, const uint8_t *__restrict__ sfb,
                     const float *__restrict__ a_global, const float *__restrict__ w_global, void *__restrict__ C,
                     int c_dtype, int M, int N, int K, int kb_per_split, float *__restrict__ partial) {
    using C_ = Cfg<BN>;
    constexpr int S = C_::S;
    constexpr uint32_t A_BYTES = C_::A_BYTES, B_BYTES = C_::B_BYTES, A_OFF = C_::A_OFF, B_OFF = C_::B_OFF,
                       SFA_OFF = C_::SFA_OFF, SFB_OFF = C_::SFB_OFF, SFA_BYTES = C_::SFA_BYTES,
                       SFB_BYTES = C_::SFB_BYTES, BAR_OFF = C_::BAR_OFF, MISC_OFF = C_::MISC_OFF;
    extern __shared__ uint8_t smem_dyn[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + BAR_OFF);
    uint64_t *empty = full + S;
    uint64_t *done = empty + S;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + MISC_OFF);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + MISC_OFF + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = blockIdx.x, nt = blockIdx.y;
    const int m0 = mt * BM, n0 = nt * BN;
    // split-K (grid z): this CTA reduces k-blocks [kb0, kb0 + nk) and, when split,
    // writes its scaled fp32 partial tile for a second kernel to sum
    const int kb0 = blockIdx.z * kb_per_split;
    const int nk = min(kb_per_split, K / BK - kb0);
    const int kchunks = K / 64;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, C_::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t tx = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
            for (int i = 0; i < nk; ++i) {
                const int s = i % S;
                if (i >= S && !wait_pf(&empty[s], (uint32_t)(((i / S) - 1) & 1), abort_flag)) break;
                const int kb = kb0 + i;
                mbar_arrive_expect_tx(&full[s], tx);
                tma_load_2d(sm + A_OFF + s * A_BYTES, &a_map, kb * (BK / 2), m0, &full[s]);
                tma_load_2d(sm + B_OFF + s * B_BYTES, &w_map, kb * (BK / 2), n0, &full[s]);
                bulk_load(sm + SFA_OFF + s * SFA_BYTES, sfa + ((size_t)mt * kchunks + 4 * kb) * SF_ATOM, SFA_BYTES,
                          &full[s]);
#pragma unroll
                for (int h = 0; h < C_::NH; ++h)  // the 128-row halves' atoms sit in separate row tiles
                    bulk_load(sm + SFB_OFF + s * SFB_BYTES + h * 4 * SF_ATOM,
                              sfb + ((size_t)(nt * C_::NH + h) * kchunks + 4 * kb) * SF_ATOM, 4 * SF_ATOM, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // Descriptors of stage 0; a stage / K step only moves the start-address
            // field (address >> 4 in the low 14 bits, never carrying out of it).
            const uint64_t a_d0 = sw128_desc(smem_u32(sm + A_OFF)), b_d0 = sw128_desc(smem_u32(sm + B_OFF));
            const uint64_t sfa_d0 = sf_desc(smem_u32(sm + SFA_OFF)), sfb_d0 = sf_desc(smem_u32(sm + SFB_OFF));
            for (int i = 0; i < nk; ++i) {
                const int s = i % S;
                if (!wait_pf(&full[s], (uint32_t)((i / S) & 1), abort_flag)) break;
                tc_fence_after();
                const uint64_t a_d = a_d0 + (uint64_t)(s * (A_BYTES >> 4)), b_d = b_d0 + (uint64_t)(s * (B_BYTES >> 4));
                const uint64_t sfa_d = sfa_d0 + (uint64_t)(s * (SFA_BYTES >> 4));
                const uint64_t sfb_d = sfb_d0 + (uint64_t)(s * (SFB_BYTES >> 4));
                const uint32_t col_a = tmem + BN + C_::SF_COLS * s, col_b = col_a + 16;
                // per K=64 step kk: A scales in 4 columns, W scales in 4 columns per 128-row half
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    tc_cp_sf(col_a + 4 * kk, sfa_d + (uint64_t)(kk * (SF_ATOM >> 4)));
#pragma unroll
                    for (int h = 0; h < C_::NH; ++h)
                        tc_cp_sf(col_b + 4 * C_::NH * kk + 4 * h, sfb_d + (uint64_t)((h * 4 + kk) * (SF_ATOM >> 4)));
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_fp4(tmem, a_d + (uint64_t)(2 * kk), b_d + (uint64_t)(2 * kk), C_::IDESC, col_a + 4 * kk,
                            col_b + 4 * C_::NH * kk, (i | kk) != 0);
                tc_commit(&empty[s]);
            }
            tc_commit(done);
        }
    } else {
        const bool ok = wait_pf(done, 0u, abort_flag);
        (void)ok;
        tc_fence_after();
        const int q = warp & 3;
        const int row = m0 + 32 * q + lane;
        const float gs = (a_global ? *a_global : 1.0f) * (w_global ? *w_global : 1.0f);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
            if (row < M) {
                const size_t base = (size_t)row * N + n0 + c0;
                if (partial || c_dtype == W4_F32) {
                    float4 *dst = reinterpret_cast<float4 *>(partial ? partial + (size_t)blockIdx.z * M * N + base
                                                                     : static_cast<float *>(C) + base);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        dst[e] = make_float4(__uint_as_float(v[4 * e]) * gs, __uint_as_float(v[4 * e + 1]) * gs,
                                             __uint_as_float(v[4 * e + 2]) * gs, __uint_as_float(v[4 * e + 3]) * gs);
                } else {
                    uint32_t p[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const float x0 = __uint_as_float(v[2 * e]) * gs, x1 = __uint_as_float(v[2 * e + 1]) * gs;
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
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C_::TMEM_COLS);
    }
}

// Persistent variant: 128 x 256 tiles in a static tile loop (tile t = blockIdx.x +
// j * gridDim.x, M fastest so a wave shares W tiles in L2), the stage ring running
// on across tiles.  One accumulator (256 TMEM columns): eight epilogue warps (two
// per TMEM lane quarter, 128 columns each) pull the whole tile into registers,
// release the accumulator to the MMA issuer at once, and only then scale and store,
// so the next tile's MMAs overlap the stores and the producer never drains.
namespace pcfg {
// warps: 0 producer, 1 MMA issuer, 2-9 epilogue, 10 scale copier
constexpr int BN = 256, S = 4, NH = 2, kEpiWarps = 8, kSfWarp = 2 + kEpiWarps, kThreadsP = (3 + kEpiWarps) * 32;
constexpr uint32_t A_BYTES = BM * BK / 2, B_BYTES = BN * BK / 2, SFA_BYTES = 4 * SF_ATOM, SFB_BYTES = NH * 4 * SF_ATOM;
constexpr uint32_t A_OFF = 0, B_OFF = A_OFF + S * A_BYTES, SFA_OFF = B_OFF + S * B_BYTES,
                   SFB_OFF = SFA_OFF + S * SFA_BYTES, BAR_OFF = SFB_OFF + S * SFB_BYTES,
                   MISC_OFF = BAR_OFF + (3 * S + 2) * 8, SMEM = MISC_OFF + 16;
// TMEM: accumulator [0, 256); stage s scales at 256 + 48 s (A 16, W 32).
constexpr uint32_t SF_COL0 = BN, SF_COLS = 16 + 16 * NH, TMEM_COLS = 512;
static_assert(SF_COL0 + S * SF_COLS <= TMEM_COLS, "TMEM plan");
constexpr uint32_t IDESC = (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}  // namespace pcfg

__global__ void __launch_bounds__(pcfg::kThreadsP, 1)
nvfp4_prefill_persistent_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap w_map,
                                const uint8_t *__restrict__ sfa, const uint8_t *__restrict__ sfb,
                                const float *__restrict__ a_global, const float *__restrict__ w_global,
                                void *__restrict__ C, int c_dtype, int M, int N, int K) {
    using namespace pcfg;
    extern __shared__ uint8_t smem_dyn[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + BAR_OFF);
    uint64_t *empty = full + S;
    uint64_t *acc_full = empty + S;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *sf_full = acc_empty + 1;  // stage s's scale atoms are in TMEM
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + MISC_OFF);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + MISC_OFF + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mtiles = (M + BM - 1) / BM;
    const int ntiles = mtiles * (N / BN);
    const int nk = K / BK;
    const int kchunks = K / 64;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kEpiWarps);  // one arrival per epilogue warp
        for (int s = 0; s < S; ++s) mbar_init(&sf_full[s], 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer: every k-block of every tile of this CTA ----------------
        if (lane == 0) {
            const uint32_t tx = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
            long g = 0;  // k-blocks issued so far (stage = g % S)
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int mt = t % mtiles, nt = t / mtiles;
                for (int i = 0; i < nk; ++i, ++g) {
                    const int s = (int)(g % S);
                    if (g >= S && !wait_pf(&empty[s], (uint32_t)(((g / S) - 1) & 1), abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], tx);
                    tma_load_2d(sm + A_OFF + s * A_BYTES, &a_map, i * (BK / 2), mt * BM, &full[s]);
                    tma_load_2d(sm + B_OFF + s * B_BYTES, &w_map, i * (BK / 2), nt * BN, &full[s]);
                    bulk_load(sm + SFA_OFF + s * SFA_BYTES, sfa + ((size_t)mt * kchunks + 4 * i) * SF_ATOM, SFA_BYTES,
                              &full[s]);
#pragma unroll
                    for (int h = 0; h < NH; ++h)
                        bulk_load(sm + SFB_OFF + s * SFB_BYTES + h * 4 * SF_ATOM,
                                  sfb + ((size_t)(nt * NH + h) * kchunks + 4 * i) * SF_ATOM, 4 * SF_ATOM, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint64_t a_d0 = sw128_desc(smem_u32(sm + A_OFF)), b_d0 = sw128_desc(smem_u32(sm + B_OFF));
            const uint64_t sfa_d0 = sf_desc(smem_u32(sm + SFA_OFF)), sfb_d0 = sf_desc(smem_u32(sm + SFB_OFF));
            long g = 0;
            int j = 0;  // local tile index
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++j) {
                if (j >= 1 && !wait_pf(acc_empty, (uint32_t)((j - 1) & 1), abort_flag)) break;
                tc_fence_after();
                for (int i = 0; i < nk; ++i, ++g) {
                    const int s = (int)(g % S);
                    // operands landed (full) and the scale copier's atoms are in TMEM (sf_full)
                    if (!wait_pf(&full[s], (uint32_t)((g / S) & 1), abort_flag) ||
                        !wait_pf(&sf_full[s], (uint32_t)((g / S) & 1), abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_d = a_d0 + (uint64_t)(s * (A_BYTES >> 4)), b_d = b_d0 + (uint64_t)(s * (B_BYTES >> 4));
                    const uint32_t col_a = tmem + SF_COL0 + SF_COLS * s, col_b = col_a + 16;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_fp4(tmem, a_d + (uint64_t)(2 * kk), b_d + (uint64_t)(2 * kk), IDESC, col_a + 4 * kk,
                                col_b + 4 * NH * kk, (i | kk) != 0);
                    tc_commit(&empty[s]);
                }
                if (!ok) break;
                tc_commit(acc_full);
            }
        }
    } else if (warp == kSfWarp) {
        // ---------------- scale copier: stage s's atoms into its TMEM columns ----------------
        // A stage's columns are rewritten only after the producer refilled the stage,
        // i.e. after the MMAs that read them committed empty[s].
        if (lane == 0) {
            const uint64_t sfa_d0 = sf_desc(smem_u32(sm + SFA_OFF)), sfb_d0 = sf_desc(smem_u32(sm + SFB_OFF));
            long g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                for (int i = 0; i < nk; ++i, ++g) {
                    const int s = (int)(g % S);
                    if (!wait_pf(&full[s], (uint32_t)((g / S) & 1), abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t sfa_d = sfa_d0 + (uint64_t)(s * (SFA_BYTES >> 4));
                    const uint64_t sfb_d = sfb_d0 + (uint64_t)(s * (SFB_BYTES >> 4));
                    const uint32_t col_a = tmem + SF_COL0 + SF_COLS * s, col_b = col_a + 16;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        tc_cp_sf(col_a + 4 * kk, sfa_d + (uint64_t)(kk * (SF_ATOM >> 4)));
#pragma unroll
                        for (int h = 0; h < NH; ++h)
                            tc_cp_sf(col_b + 4 * NH * kk + 4 * h, sfb_d + (uint64_t)((h * 4 + kk) * (SF_ATOM >> 4)));
                    }
                    tc_commit(&sf_full[s]);
                }
            }
            // nothing of this warp may still be in flight when TMEM is freed
            if (g > 0 && !mbar_wait_bounded(&sf_full[(int)((g - 1) % S)], (uint32_t)(((g - 1) / S) & 1)))
                atomicExch(&g_fp4pf_timeout, 1u);
        }
    } else {
        // ---------------- epilogue warps 2-9: lane quarter warp % 4, column half (warp - 2) / 4 ----------------
        const int q = warp & 3, ch = (warp - 2) >> 2;
        const float gs = (a_global ? *a_global : 1.0f) * (w_global ? *w_global : 1.0f);
        int j = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++j) {
            if (!__all_sync(0xffffffffu, wait_pf(acc_full, (uint32_t)(j & 1), abort_flag))) break;
            tc_fence_after();
            uint32_t v[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c)
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(128 * ch + 32 * c), v[c]);
            tc_fence_before();  // TMEM reads done: the accumulator may be overwritten
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
            const int mt = t % mtiles, nt = t / mtiles;
            const int row = mt * BM + 32 * q + lane;
            if (row < M) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const size_t base = (size_t)row * N + nt * BN + 128 * ch + 32 * c;
                    if (c_dtype == W4_F32) {
                        float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(C) + base);
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            dst[e] = make_float4(__uint_as_float(v[c][4 * e]) * gs, __uint_as_float(v[c][4 * e + 1]) * gs,
                                                 __uint_as_float(v[c][4 * e + 2]) * gs,
                                                 __uint_as_float(v[c][4 * e + 3]) * gs);
                    } else {
                        uint32_t p[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const float x0 = __uint_as_float(v[c][2 * e]) * gs, x1 = __uint_as_float(v[c][2 * e + 1]) * gs;
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
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace fp4pf

namespace fp4pf {
template <int BN>
static int launch(const CUtensorMap &a_map, const CUtensorMap &w_map, const uint8_t *sfa, const uint8_t *sfb,
                  const float *a_global, const float *w_global, void *c, int c_dtype, int M, int N, int K,
                  int ksplit, float *partial, cudaStream_t st) {
    const size_t smem = Cfg<BN>::SMEM + 1024;
    auto kern = nvfp4_prefill_kernel<BN>;
    {
        static std::mutex mu;
        static bool set_dev[128] = {};
        int dev = 0;
        W4_CUDA_TRY(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lk(mu);
        if (dev < 128 && !set_dev[dev]) {
            W4_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            set_dev[dev] = true;
        }
    }
    const int nk = K / BK;
    const int kb_per_split = (nk + ksplit - 1) / ksplit;
    ksplit = (nk + kb_per_split - 1) / kb_per_split;  // every split gets at least one k-block
    dim3 grid((M + BM - 1) / BM, N / BN, ksplit), block(kThreads);
    kern<<<grid, block, smem, st>>>(a_map, w_map, sfa, sfb, a_global, w_global, c, c_dtype, M, N, K, kb_per_split,
                                    ksplit > 1 ? partial : nullptr);
    W4_LAUNCH_CHECK();
    if (ksplit > 1) return splitk_reduce(partial, ksplit, (long)M * N, c, c_dtype, st);  // N % 128 == 0
    return W4_OK;
}

// K splits for grids that fill at most half the SMs (the non-persistent form):
// up to one wave, at least two k-blocks per split, at most 4 (each split adds an
// M x N fp32 partial to write and read back).
static int ksplit_for(int M, int N, int K) {
    const bool wide = N % 256 == 0;
    const long tiles = (long)((M + BM - 1) / BM) * (N / (wide ? 256 : 128));
    const long nsm = num_sms();
    if (2 * tiles > nsm) return 1;
    long ks = nsm / tiles;
    if (ks > (K / BK) / 2) ks = (K / BK) / 2;
    if (ks > 4) ks = 4;
    return ks < 1 ? 1 : (int)ks;
}
}  // namespace fp4pf

namespace fp4pf {
static int launch_persistent(const CUtensorMap &a_map, const CUtensorMap &w_map, const uint8_t *sfa,
                             const uint8_t *sfb, const float *a_global, const float *w_global, void *c, int c_dtype,
                             int M, int N, int K, cudaStream_t st) {
    const size_t smem = pcfg::SMEM + 1024;
    auto kern = nvfp4_prefill_persistent_kernel;
    {
        static std::mutex mu;
        static bool set_dev[128] = {};
        int dev = 0;
        W4_CUDA_TRY(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lk(mu);
        if (dev < 128 && !set_dev[dev]) {
            W4_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            set_dev[dev] = true;
        }
    }
    const int tiles = (M + BM - 1) / BM * (N / pcfg::BN);
    const int grid = tiles < num_sms() ? tiles : num_sms();
    kern<<<grid, pcfg::kThreadsP, smem, st>>>(a_map, w_map, sfa, sfb, a_global, w_global, c, c_dtype, M, N, K);
    W4_LAUNCH_CHECK();
    return W4_OK;
}
}  // namespace fp4pf

static size_t split_bytes(int M, int N, int K) {
    if (K % fp4pf::BK || N % 128) return 0;
    const int ks = fp4pf::ksplit_for(M, N, K);
    return ks > 1 ? align256((size_t)ks * M * N * sizeof(float)) : 0;
}

size_t nvfp4_prefill_workspace(int M, int N, int K) {
    const size_t mp = (size_t)(M + 127) / 128 * 128, np = (size_t)(N + 127) / 128 * 128;
    return align256(mp * K / 2) + align256(mp * (K / 16)) + align256(np * (K / 16)) + split_bytes(M, N, K);
}

// The block-scaled GEMM on activations already quantised: codes u8 [rows, K/2]
// and scale atoms for rows = M rounded up to 128 (padding rows with zero
// scales); weight scales rearranged into atoms in the workspace unless
// w_sf_atoms.  -1: shape not handled.
int nvfp4_prefill_q(const uint8_t *codes, const uint8_t *sfa, const float *a_global, const uint8_t *w_nk,
                    const uint8_t *w_sf, bool w_sf_atoms, const float *w_global, void *c, int c_dtype, int M, int N,
                    int K, void *workspace, cudaStream_t st) {
    using namespace fp4pf;
    if (K % BK || N % 128 || c_dtype == W4_E4M3) return -1;
    const size_t mp = (size_t)(M + 127) / 128 * 128;
    const uint8_t *sfb = w_sf;
    char *wsb = static_cast<char *>(workspace);
    if (!w_sf_atoms) {
        uint8_t *t = reinterpret_cast<uint8_t *>(wsb);
        const int rc = nvfp4_sf_atoms(w_sf, N, K / 16, 1, N, t, st);
        if (rc) return rc;
        sfb = t;
        wsb += align256((size_t)(N + 127) / 128 * 128 * (K / 16));
    }
    float *partial = reinterpret_cast<float *>(wsb);  // split-K partials (split_bytes)
    CUtensorMap a_map, w_map;
    // 256-wide tiles: persistent when there are more tiles than SMs, one tile per
    // CTA otherwise; 128-wide tiles when N is not a multiple of 256.
    const bool wide = N % 256 == 0;
    const long tiles256 = (long)((M + BM - 1) / BM) * (N / 256);
    const bool persistent = wide && tiles256 > num_sms();
    const int bn = wide ? 256 : 128;
    if (!make_map_2d(&a_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, (uint64_t)K / 2, mp, (uint64_t)K / 2, BK / 2, BM,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&w_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_nk, (uint64_t)K / 2, N, (uint64_t)K / 2, BK / 2, bn,
                     CU_TENSOR_MAP_SWIZZLE_128B))
        return -1;
    if (persistent) return launch_persistent(a_map, w_map, sfa, sfb, a_global, w_global, c, c_dtype, M, N, K, st);
    const int ks = workspace ? ksplit_for(M, N, K) : 1;
    return wide ? launch<256>(a_map, w_map, sfa, sfb, a_global, w_global, c, c_dtype, M, N, K, ks, partial, st)
                : launch<128>(a_map, w_map, sfa, sfb, a_global, w_global, c, c_dtype, M, N, K, ks, partial, st);
}

size_t nvfp4_prefill_q_workspace(int M, int N, int K, bool scale_atoms_needed) {
    const size_t np = (size_t)(N + 127) / 128 * 128;
    return (scale_atoms_needed ? align256(np * (K / 16)) : 0) + split_bytes(M, N, K);
}

// A bf16 [M,K] -> NVFP4 codes + scale atoms in the workspace, then nvfp4_prefill_q.
int nvfp4_prefill(const uint16_t *a, const float *a_global, const uint8_t *w_nk, const uint8_t *w_sf,
                  bool w_sf_atoms, const float *w_global, void *c, int c_dtype, int M, int N, int K,
                  void *workspace, cudaStream_t st) {
    using namespace fp4pf;
    if (K % BK || N % 128 || c_dtype == W4_E4M3) return -1;
    char *ws = static_cast<char *>(workspace);
    const size_t mp = (size_t)(M + 127) / 128 * 128;
    uint8_t *codes = reinterpret_cast<uint8_t *>(ws);  // rows padded to the 128-row tile; the pad
    ws += align256(mp * K / 2);                         // rows' scales are 0
    uint8_t *sfa = reinterpret_cast<uint8_t *>(ws);
    ws += align256(mp * (K / 16));
    const int rc = nvfp4_quant_act_atoms(a, M, K, a_global, codes, sfa, st);
    if (rc) return rc;
    return nvfp4_prefill_q(codes, sfa, a_global, w_nk, w_sf, w_sf_atoms, w_global, c, c_dtype, M, N, K, ws, st);
}

int take_fp4_prefill_wait_status() {
    unsigned int v = 0;
    W4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_fp4pf_timeout, sizeof(v)));
    if (v) {
        const unsigned int zero = 0;
        W4_CUDA_TRY(cudaMemcpyToSymbol(g_fp4pf_timeout, &zero, sizeof(zero)));
        set_error("a device-side wait expired in the NVFP4 prefill GEMM");
        return W4_ERR_TIMEOUT;
    }
    return W4_OK;
}

}  // namespace w4
