// gptq_tma.cu -- GPTQ int4 decode GEMM with TMA-streamed weights (sm_100a).
//
// Same math and register mapping as the batched decode kernel in gptq.cu (swap-AB
// m16n8k16 MMAs, exact (q - zero) in 16-bit floats, per-group fp32 scaling), but
// the weights reach shared memory through the tensor-memory accelerator.  A CTA
// owns 32 output columns; its W consumer warps split K evenly and each owns a
// ring of kTmaStages stages; a stage is kVps groups (qweight rows x 32 columns
// as a 128-byte-wide, 128-byte-swizzled box) plus those groups' scale rows and
// zero rows, all completing on one "full" mbarrier.  One extra producer warp
// issues every copy and refills a stage when its consumer arrives on the
// stage's "empty" mbarrier, so the consumers' instruction stream is only the
// dequantisation and the MMAs.  Every wait is bounded: on expiry the waiting
// warp stops, a device status word is set and w4_check_device_status()
// reports W4_ERR_TIMEOUT.  No copy uses multicast.
//
// Bulk copies move whole tiles per instruction without holding registers, so
// each SM keeps >100 KB of weight reads in flight while its warps compute.

#include <mutex>
#include <type_traits>

#include "tma_util.cuh"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

static __device__ unsigned int g_wait_timeout;  // a bounded wait expired (sticky until read)
static __device__ unsigned int g_tpf_timeout;   // a peer's tile never arrived in the fused all-reduce

constexpr unsigned long long kPeerWaitNs = 500ull * 1000 * 1000;  // 500 ms

__device__ __forceinline__ void peer_st_release(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t peer_ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

constexpr int kTmaStages = 3;   // ring depth per consumer warp
constexpr int kVps = 2;         // virtual groups per stage
constexpr int kTmaMaxWarps = 8; // consumer warps per CTA (one more warp produces)
// Register cap: 4 CTAs of 4 warps (the usual one-wave shape) must fit an SM's
// 64K registers, so 128 at most.
constexpr int kTmaMaxRegs = 128;

// Shared-memory ring of one consumer warp (byte offsets from its 1024-aligned
// base; every tensor-copy destination is 128-byte aligned, the swizzled tiles
// 1024):  S qweight stages | S activation stages | S constant stages (scales at
// +0, zeros at +128) | S full + S empty mbarriers | the warp's reduction slot.
struct RingLayout {
    uint32_t qw_stage, act_stage, act, cst, bars, red, total;
    __host__ __device__ RingLayout(int qw_bytes, int act_bytes, int red_bytes) {
        qw_stage = qw_bytes;
        act_stage = (act_bytes + 1023) & ~1023;
        act = kTmaStages * qw_stage;
        cst = act + kTmaStages * act_stage;
        bars = cst + kTmaStages * 256;
        red = (bars + 2 * kTmaStages * 8 + 127) & ~127u;
        total = (red + red_bytes + 1023) & ~1023u;
    }
};

template <typename T> struct DeqT;
template <> struct DeqT<__nv_bfloat16> {
    static constexpr uint32_t kMagic = 0x43004300u, kMagicHalf = 0x4300u;  // 128 + q
    static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
        __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162 *>(&a), *reinterpret_cast<__nv_bfloat162 *>(&b));
        return *reinterpret_cast<uint32_t *>(&r);
    }
};
template <> struct DeqT<__half> {
    static constexpr uint32_t kMagic = 0x64006400u, kMagicHalf = 0x6400u;  // 1024 + q
    static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
        __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
        return *reinterpret_cast<uint32_t *>(&r);
    }
};

// Lane quad g reads 16-byte chunk sigma(g) = (0,4,1,5,2,6,3,7)[g] of each 128-byte
// row: with the 128-byte swizzle (chunk ^= row % 8) the 8 lanes of every
// shared-load phase then hit 8 distinct bank groups.
__device__ __forceinline__ int sigma(int g) { return (g >> 1) | ((g & 1) << 2); }

// ACT: activations arrive by TMA with the stage (rows of up to 8*NT tokens x the
// stage's k range, a 3-D box over [K/64][M][64] so each 64-k row segment is one
// 128-byte-swizzled line); otherwise each lane loads them from global memory one
// step ahead.
//
// AR: the row-parallel form.  Instead of storing its tile, a CTA pushes the fp32
// partial tile into slot [parity][rank] of every rank's peer buffer (NVLink
// stores), fences at system scope, raises its flag [parity][cta][rank] on every
// rank, waits (bounded) until the same CTA of every rank has raised its flag
// here, and stores the sum of the nranks partials in rank order (the same bits
// on every rank).  The call's sequence number v (parity v & 1) is read from the
// communicator's control word at the epilogue; the last CTA to finish advances
// it, so graph replays stay in step.  Launched cooperatively: every CTA of the
// grid is resident, so each one's peer counterpart runs as well.
template <typename T, int NT, int GSTEPS, bool ACT, bool AR>
__global__ void __maxnreg__(kTmaMaxRegs)
gptq_gemv_tma_kernel(const __grid_constant__ CUtensorMap qw_map, const __grid_constant__ CUtensorMap sc_map,
                     const __grid_constant__ CUtensorMap zr_map, const __grid_constant__ CUtensorMap act_map,
                     int has_z, const T *__restrict__ A, void *__restrict__ C, int c_dtype, int M, int N, int K,
                     int zero_offset, int stages_all, int act_rows, int pre, const __grid_constant__ PeerReduce pr) {
    constexpr int S = kTmaStages;
    constexpr int NE = 2 * NT * 4;
    constexpr int ROWS = 4 * GSTEPS;           // qweight rows per group
    constexpr int SSTEPS = kVps * GSTEPS;      // 32-k steps per stage
    extern __shared__ uint8_t smem_dyn[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int W = (blockDim.x >> 5) - 1;        // consumer warps; warp W produces
    const RingLayout L(kVps * ROWS * 128, ACT ? act_rows * SSTEPS * 64 : 0, NE * 32 * 4);
    const int n0 = blockIdx.y * 32;
    const int tok0 = blockIdx.x * 8 * NT;
    // Split K across the CTAs of a cluster (grid z): this CTA owns stages
    // [zb, zb + stages_total) of the stages_all stages of K.
    const int zb = (int)(blockIdx.z * (unsigned)stages_all / gridDim.z);
    const int stages_total = (int)((blockIdx.z + 1) * (unsigned)stages_all / gridDim.z) - zb;
    // Warp w consumes stages [w*stages_total/W, (w+1)*stages_total/W) of them; a
    // stage is kVps whole groups.

    if (warp == W) {  // ---------------- producer warp ----------------
        if (lane == 0) {
            for (int w = 0; w < W; ++w) {
                uint64_t *bars = reinterpret_cast<uint64_t *>(base + (size_t)w * L.total + L.bars);
                for (int i = 0; i < 2 * S; ++i) mbar_init(&bars[i], 1);
            }
            fence_mbar_init();
        }
    }
    __syncthreads();  // barriers initialised before anyone waits on them
    if (warp == W) {
        if (lane == 0) {
            const uint32_t tx = kVps * (ROWS * 128 + 64 + (has_z ? 16 : 0)) + (ACT ? act_rows * SSTEPS * 64 : 0);
            bool ok = true;
            const int most = (stages_total + W - 1) / W;
            // pre: the weight operands of the first ring fill are requested before
            // the previous kernel on the stream has completed (static weights).
            const int pf = pre ? (most < S ? most : S) : 0;
            for (int it = 0; it < pf; ++it)
                for (int w = 0; w < W; ++w) {
                    const int sb = w * stages_total / W, se = (w + 1) * stages_total / W;
                    if (sb + it >= se) continue;
                    uint8_t *r = base + (size_t)w * L.total;
                    uint64_t *full = reinterpret_cast<uint64_t *>(r + L.bars) + it;
                    const int vg = (zb + sb + it) * kVps;
                    mbar_arrive_expect_tx(full, tx);
                    tma_load_2d(r + it * L.qw_stage, &qw_map, n0, vg * ROWS, full);
                    tma_load_2d(r + L.cst + it * 256, &sc_map, n0, vg, full);
                    if (has_z) tma_load_2d(r + L.cst + it * 256 + 128, &zr_map, n0 / 8, vg, full);
                }
            grid_dep_wait();  // activations are the previous kernel's output
            for (int it = 0; it < most && ok; ++it) {
                const int s = it % S;
                for (int w = 0; w < W && ok; ++w) {
                    const int sb = w * stages_total / W, se = (w + 1) * stages_total / W;
                    if (sb + it >= se) continue;
                    uint8_t *r = base + (size_t)w * L.total;
                    uint64_t *full = reinterpret_cast<uint64_t *>(r + L.bars) + s;
                    uint64_t *empty = full + S;
                    const int vg = (zb + sb + it) * kVps;  // first group of the stage
                    if (it >= pf) {
                        if (it >= S && !mbar_wait_bounded(empty, (uint32_t)(((it / S) - 1) & 1))) {
                            atomicExch(&g_wait_timeout, 1u);
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(full, tx);
                        tma_load_2d(r + s * L.qw_stage, &qw_map, n0, vg * ROWS, full);
                        tma_load_2d(r + L.cst + s * 256, &sc_map, n0, vg, full);
                        if (has_z) tma_load_2d(r + L.cst + s * 256 + 128, &zr_map, n0 / 8, vg, full);
                    }
                    if (ACT) tma_load_3d(r + L.act + s * L.act_stage, &act_map, 0, tok0, (vg * ROWS) / 8, full);  // 64-k line of the stage
                }
            }
        }
        __syncwarp();
        grid_dep_launch();  // every copy is issued: the next decode GEMM may be scheduled
        if (gridDim.z > 1) {  // meet the consumers at the cluster reduction's two barriers
            cluster_sync_all();
            cluster_sync_all();
        }
        return;  // consumers wait for every copy this warp issued
    }
    grid_dep_wait();  // nothing below touches global memory before the previous kernel completed

    // ---------------- consumer warps ----------------
    uint8_t *ring = base + (size_t)warp * L.total;
    uint64_t *fullb = reinterpret_cast<uint64_t *>(ring + L.bars);
    float *red = reinterpret_cast<float *>(ring + L.red);
    const int g = lane >> 2, t = lane & 3, sg = sigma(g);
    const int sbeg = warp * stages_total / W;
    const int nstages = (warp + 1) * stages_total / W - sbeg;
    const int nsteps = nstages * SSTEPS;
    // Register-path activations (ACT == false).
    const T *ap[NT];
    bool av[NT];
    uint4 xa[NT];
    // TMA-path activations: this lane's 16-byte chunk of step j (line kc = j/2,
    // chunk 4*(j%2) + t) for token row 8*nt + g; rows past the box read row 0
    // (their outputs are discarded).
    uint32_t aoff[ACT ? SSTEPS : 1][NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        if constexpr (ACT) {
            const int row = (nt * 8 + g) < act_rows ? nt * 8 + g : 0;
#pragma unroll
            for (int j = 0; j < SSTEPS; ++j) {
                const int line = (j >> 1) * act_rows + row;
                aoff[j][nt] = line * 128 + (((4 * (j & 1) + t) ^ (line & 7)) << 4);
            }
        } else {
            const int tok = tok0 + nt * 8 + g;
            av[nt] = tok < M;
            ap[nt] = A + (size_t)(av[nt] ? tok : 0) * K + (size_t)((zb + sbeg) * kVps * ROWS + t) * 8;
            xa[nt] = (av[nt] && nsteps > 0) ? __ldg(reinterpret_cast<const uint4 *>(ap[nt])) : make_uint4(0, 0, 0, 0);
            ap[nt] += 32;
        }
    }
    // This lane's 16-byte chunk in qweight row 4i + t of group vv of a stage; the
    // 128-byte swizzle XORs the chunk index with the row index mod 8.
    uint32_t roff[kVps][GSTEPS];
#pragma unroll
    for (int vv = 0; vv < kVps; ++vv)
#pragma unroll
        for (int i = 0; i < GSTEPS; ++i) {
            const int r = vv * ROWS + 4 * i + t;
            roff[vv][i] = r * 128 + ((sg ^ (r & 7)) << 4);
        }
    const uint32_t zsh = 16 * (sg & 1);
    const uint32_t zbase = DeqT<T>::kMagicHalf + (has_z ? (uint32_t)zero_offset : 0u);

    float facc[2][NT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) facc[a][b][i] = 0.f;

    uint32_t parity = 0;
    bool ok = true;
    for (int it0 = 0; it0 < nstages && ok; it0 += S, parity ^= 1u) {
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const int it = it0 + s;
            if (it < nstages && ok) {
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(&fullb[s], parity))) {
                    if (lane == 0) atomicExch(&g_wait_timeout, 1u);
                    ok = false;  // stop; this warp still meets the others below
                } else {
                    const uint8_t *qws = ring + s * L.qw_stage;
                    const uint8_t *acts = ring + L.act + s * L.act_stage;
                    const uint8_t *cst = ring + L.cst + s * 256;
#pragma unroll
                    for (int vv = 0; vv < kVps; ++vv) {
                        const uint2 sw = *reinterpret_cast<const uint2 *>(cst + vv * 64 + 8 * sg);
                        const uint32_t zw = has_z ? (*reinterpret_cast<const uint32_t *>(cst + 128 + vv * 16 + 4 * (sg >> 1)) >> zsh)
                                                  : 0x8888u;
                        uint32_t zc[4];
#pragma unroll
                        for (int c = 0; c < 4; ++c) zc[c] = (zbase + ((zw >> (4 * c)) & 15u)) * 0x00010001u;
                        float gacc[2][NT][4];
#pragma unroll
                        for (int a = 0; a < 2; ++a)
#pragma unroll
                            for (int b = 0; b < NT; ++b)
#pragma unroll
                                for (int i = 0; i < 4; ++i) gacc[a][b][i] = 0.f;
#pragma unroll
                        for (int i = 0; i < GSTEPS; ++i) {
                            const int j = vv * GSTEPS + i;  // step within the stage
                            const uint4 wv = *reinterpret_cast<const uint4 *>(qws + roff[vv][i]);
                            uint32_t bf[NT][2][2];
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt) {
                                uint4 x;
                                if constexpr (ACT) {
                                    x = *reinterpret_cast<const uint4 *>(acts + aoff[j][nt]);
                                } else {
                                    x = xa[nt];
                                    if (av[nt] && it * SSTEPS + j + 1 < nsteps)
                                        xa[nt] = __ldg(reinterpret_cast<const uint4 *>(ap[nt]));
                                    ap[nt] += 32;
                                }
                                bf[nt][0][0] = __byte_perm(x.x, x.z, 0x5410);
                                bf[nt][0][1] = __byte_perm(x.x, x.z, 0x7632);
                                bf[nt][1][0] = __byte_perm(x.y, x.w, 0x5410);
                                bf[nt][1][1] = __byte_perm(x.y, x.w, 0x7632);
                            }
                            const uint32_t wc[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                            for (int mt = 0; mt < 2; ++mt) {
                                const uint32_t lo = wc[2 * mt], hi = wc[2 * mt + 1];
#pragma unroll
                                for (int q = 0; q < 2; ++q) {
                                    const uint32_t a0 = DeqT<T>::sub(lop3_and_or(lo >> (8 * q), 0x000F000Fu, DeqT<T>::kMagic), zc[2 * mt]);
                                    const uint32_t a1 = DeqT<T>::sub(lop3_and_or(hi >> (8 * q), 0x000F000Fu, DeqT<T>::kMagic), zc[2 * mt + 1]);
                                    const uint32_t a2 = DeqT<T>::sub(lop3_and_or(lo >> (8 * q + 4), 0x000F000Fu, DeqT<T>::kMagic), zc[2 * mt]);
                                    const uint32_t a3 = DeqT<T>::sub(lop3_and_or(hi >> (8 * q + 4), 0x000F000Fu, DeqT<T>::kMagic), zc[2 * mt + 1]);
#pragma unroll
                                    for (int nt = 0; nt < NT; ++nt)
                                        mma_16816<T>(gacc[mt][nt], a0, a1, a2, a3, bf[nt][q][0], bf[nt][q][1]);
                                }
                            }
                        }
                        const float2 s01 = __half22float2(*reinterpret_cast<const __half2 *>(&sw.x));
                        const float2 s23 = __half22float2(*reinterpret_cast<const __half2 *>(&sw.y));
                        const float sc[4] = {s01.x, s01.y, s23.x, s23.y};
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
                    __syncwarp();  // every lane is done with stage s
                    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&fullb[S + s])) : "memory");
                }
            }
        }
    }

    // ---- K-split reduction across the W consumer warps ----
    // The next decode GEMM may be scheduled once every thread of every CTA is here
    // (late, so its CTAs take the slots this grid frees, evenly).
    grid_dep_launch();
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[((mt * NT + nt) * 4 + i) * 32 + lane] = facc[mt][nt][i];
    asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");  // consumers only
    if constexpr (!AR) {
        if (gridDim.z == 1) {
            for (int idx = threadIdx.x; idx < NE * 32; idx += W * 32) {
                float val = 0.f;
                for (int w = 0; w < W; ++w) val += reinterpret_cast<const float *>(base + (size_t)w * L.total + L.red)[idx];
                const int e = idx >> 5, l = idx & 31;
                const int mt = e / (NT * 4), nt = (e / 4) % NT, i = e & 3;
                const int col = n0 + 4 * sigma(l >> 2) + 2 * mt + (i >> 1);
                const int tok = tok0 + nt * 8 + 2 * (l & 3) + (i & 1);
                if (tok < M) store_out(C, c_dtype, (size_t)tok * N + col, val);
            }
        } else {
            // K split over the cluster: each CTA leaves its partial tile in its own
            // shared memory; CTA r of the cluster sums elements r, r + ks, ... over
            // the cluster's CTAs in rank order (DSMEM loads) and stores them.
            float *fin = reinterpret_cast<float *>(base + (size_t)W * L.total);
            for (int idx = threadIdx.x; idx < NE * 32; idx += W * 32) {
                float val = 0.f;
                for (int w = 0; w < W; ++w) val += reinterpret_cast<const float *>(base + (size_t)w * L.total + L.red)[idx];
                fin[idx] = val;
            }
            cluster_sync_all();
            const int ks = (int)gridDim.z, cr = (int)cluster_rank();
            for (int idx = cr + ks * (int)threadIdx.x; idx < NE * 32; idx += ks * W * 32) {
                float val = 0.f;
                for (int c = 0; c < ks; ++c) val += ld_cluster_f32(fin + idx, (uint32_t)c);
                const int e = idx >> 5, l = idx & 31;
                const int mt = e / (NT * 4), nt = (e / 4) % NT, i = e & 3;
                const int col = n0 + 4 * sigma(l >> 2) + 2 * mt + (i >> 1);
                const int tok = tok0 + nt * 8 + 2 * (l & 3) + (i & 1);
                if (tok < M) store_out(C, c_dtype, (size_t)tok * N + col, val);
            }
            cluster_sync_all();  // no CTA leaves while another still reads its tile
        }
    } else {
        // tile rows of 32 fp32 outputs, 16-byte vectors to and from the peer slots
        __shared__ __align__(16) float tile[16][32];
        __shared__ uint32_t v_sh;
        const int nr = pr.nranks, me = pr.rank;
        const int b = blockIdx.y * gridDim.x + blockIdx.x;
        const int rows = min(8 * NT, M - tok0);
        uint32_t *ctrl = reinterpret_cast<uint32_t *>(pr.buf[me] + pr.ctrl_off);
        if (threadIdx.x == 0) v_sh = *reinterpret_cast<volatile uint32_t *>(ctrl) + 1;
        for (int idx = threadIdx.x; idx < NE * 32; idx += W * 32) {
            float val = 0.f;
            for (int w = 0; w < W; ++w) val += reinterpret_cast<const float *>(base + (size_t)w * L.total + L.red)[idx];
            const int e = idx >> 5, l = idx & 31;
            const int mt = e / (NT * 4), nt = (e / 4) % NT, i = e & 3;
            tile[nt * 8 + 2 * (l & 3) + (i & 1)][4 * sigma(l >> 2) + 2 * mt + (i >> 1)] = val;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
        const uint32_t v = v_sh;
        const int par = v & 1;
        const size_t slot0 = pr.data_off + (size_t)(par * nr) * pr.slot_bytes;  // slot [par][0]
        // 1. push the fp32 partial tile into slot [par][me] of every rank
        for (int q = threadIdx.x; q < rows * 8; q += W * 32) {
            const int r = q >> 3, c4 = (q & 7) * 4;
            const float4 x = *reinterpret_cast<const float4 *>(&tile[r][c4]);
            const size_t off = slot0 + (size_t)me * pr.slot_bytes + ((size_t)(tok0 + r) * N + n0 + c4) * 4;
            for (int p = 0; p < nr; ++p) *reinterpret_cast<float4 *>(pr.buf[p] + off) = x;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
        // 2. flag this CTA's push on every rank (the system fence and release are
        // cumulative over the CTA barrier above), then wait for every rank's push here
        if (threadIdx.x < nr) {
            __threadfence_system();
            uint32_t *fl = reinterpret_cast<uint32_t *>(pr.buf[threadIdx.x] + pr.flags_off);
            peer_st_release(fl + ((size_t)par * pr.max_ctas + b) * 8 + me, v);
            const uint32_t *mine = reinterpret_cast<const uint32_t *>(pr.buf[me] + pr.flags_off) +
                                   ((size_t)par * pr.max_ctas + b) * 8 + threadIdx.x;
            if (peer_ld_acquire(mine) != v) {
                const unsigned long long t0 = global_ns();
                while (peer_ld_acquire(mine) != v) {
                    if (global_ns() - t0 > kPeerWaitNs) {
                        atomicExch(&g_tpf_timeout, 1u);
                        break;
                    }
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
        // 3. sum the partials in rank order
        for (int q = threadIdx.x; q < rows * 8; q += W * 32) {
            const int r = q >> 3, c4 = (q & 7) * 4;
            const size_t e0 = (size_t)(tok0 + r) * N + n0 + c4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int p = 0; p < nr; ++p) {
                const float4 x = __ldcg(reinterpret_cast<const float4 *>(pr.buf[me] + slot0 + (size_t)p * pr.slot_bytes + e0 * 4));
                acc.x += x.x, acc.y += x.y, acc.z += x.z, acc.w += x.w;
            }
            store_out(C, c_dtype, e0, acc.x);
            store_out(C, c_dtype, e0 + 1, acc.y);
            store_out(C, c_dtype, e0 + 2, acc.z);
            store_out(C, c_dtype, e0 + 3, acc.w);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
        // 4. the last CTA of the grid advances the call sequence
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(ctrl + 1, 1u) == gridDim.x * gridDim.y - 1) {
                *reinterpret_cast<volatile uint32_t *>(ctrl + 1) = 0;
                __threadfence();
                *reinterpret_cast<volatile uint32_t *>(ctrl) = v;
            }
        }
    }
}

// ---- host side ----
template <typename T, int NT, int GSTEPS, bool ACT, bool AR>
static int launch_tma_t(const void *a, const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                        void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset, const PeerReduce *pr,
                        cudaStream_t st) {
    constexpr int NE = 2 * NT * 4;
    constexpr int SSTEPS = kVps * GSTEPS;
    if (gs != 32 * GSTEPS) return -1;  // one real group per virtual group only
    const int nsm = num_sms();
    const int nchunk = N / 32;
    const int mblocks = (M + 8 * NT - 1) / (8 * NT);
    const int nvg = K / gs;
    if (nvg % kVps) return -1;  // whole stages only
    const int stages_total = nvg / kVps;
    const int act_rows = M < 8 * NT ? M : 8 * NT;
    const RingLayout lay(kVps * 4 * GSTEPS * 128, ACT ? act_rows * SSTEPS * 64 : 0, NE * 32 * 4);
    const size_t per_warp = lay.total;
    // Consumer warps per CTA (the K split): as many as fit when the whole grid is
    // resident in one wave (ctas_per_sm CTAs sharing an SM's 224 KB), at most
    // one per stage.
    const long ctas = (long)nchunk * mblocks;
    // Fewer column tiles than two per SM: split K over a cluster of ks CTAs per
    // tile (reduced through distributed shared memory), so more warps share the
    // stages and the tiles spread evenly over the SMs.
    int ks = 1;
    if (!AR && ctas < 2L * nsm) {
        ks = (int)((2L * nsm + ctas - 1) / ctas);
        if (ks > 4) ks = 4;
        if (ks > stages_total) ks = stages_total;
    }
    const size_t fin_bytes = ks > 1 ? (size_t)NE * 32 * 4 : 0;
    const long ctas_per_sm = (ctas * ks + nsm - 1) / nsm;
    long fit = ((224L * 1024) / ctas_per_sm - 1024 - (long)fin_bytes) / (long)per_warp;
    // the register file must hold ctas_per_sm CTAs of W + 1 warps as well
    const long fit_regs = 65536L / (ctas_per_sm * 32L * kTmaMaxRegs) - 1;
    if (fit_regs < fit) fit = fit_regs;
    int W = (int)(fit < 1 ? 1 : (fit > kTmaMaxWarps ? kTmaMaxWarps : fit));
    if (W > stages_total / ks) W = stages_total / ks;  // every warp of every CTA gets a stage
    const CUtensorMapDataType adt =
        std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap qw_map, sc_map, zr_map, act_map;
    if (!make_map_2d(&qw_map, CU_TENSOR_MAP_DATA_TYPE_INT32, qweight, N, K / 8, (uint64_t)N * 4, 32,
                     kVps * 4 * GSTEPS, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&sc_map, CU_TENSOR_MAP_DATA_TYPE_UINT16, scales, N, K / gs, (uint64_t)N * 2, 32, kVps,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return -1;
    const int has_z = qzeros != nullptr;
    if (has_z) {
        if (!make_map_2d(&zr_map, CU_TENSOR_MAP_DATA_TYPE_INT32, qzeros, N / 8, K / gs, (uint64_t)N / 2, 4, kVps,
                         CU_TENSOR_MAP_SWIZZLE_NONE))
            return -1;
    } else {
        zr_map = sc_map;  // unused
    }
    if (ACT) {
        if (K % 64 || !make_act_map(&act_map, adt, a, M, K, act_rows, SSTEPS / 2)) return -1;
    } else {
        act_map = sc_map;  // unused
    }
    auto kern = gptq_gemv_tma_kernel<T, NT, GSTEPS, ACT, AR>;
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
    const size_t smem = 1024 + (size_t)W * per_warp + fin_bytes;
    if (smem > 220 * 1024) return -1;
    dim3 grid(mblocks, nchunk, ks), block(32 * (W + 1));
    if constexpr (AR) {
        // every CTA must be resident at once (each waits for its peers' counterpart)
        if (ctas > pr->max_ctas || (size_t)M * N * 4 > pr->slot_bytes) return -1;
        int per_sm = 0;
        W4_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (int)block.x, smem));
        if ((long)per_sm * nsm < ctas) return -1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid;
        cfg.blockDim = block;
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeCooperative;
        at[0].val.cooperative = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        W4_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, qw_map, sc_map, zr_map, act_map, has_z, static_cast<const T *>(a),
                                       c, c_dtype, M, N, K, zero_offset, stages_total, act_rows, 0, *pr));
    } else {
        const int pre = launch_overlap() == W4_OVERLAP_STATIC_WEIGHTS;
        const PeerReduce none{};
        W4_CUDA_TRY(launch_decode(kern, grid, block, smem, st, (unsigned)ks, qw_map, sc_map, zr_map, act_map, has_z,
                                  static_cast<const T *>(a), c, c_dtype, M, N, K, zero_offset, stages_total, act_rows,
                                  pre, none));
    }
    return W4_OK;
}

template <typename T, int NT, bool AR>
static int launch_tma_nt(const void *a, const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                         void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset, const PeerReduce *pr,
                         cudaStream_t st) {
    constexpr bool ACT = NT == 1;  // staged activations fit the ring only for <= 8 tokens
    if (gs == 128)
        return launch_tma_t<T, NT, 4, ACT, AR>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, pr, st);
    if (gs == 64)
        return launch_tma_t<T, NT, 2, ACT, AR>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, pr, st);
    if (gs == 32)
        return launch_tma_t<T, NT, 1, ACT, AR>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, pr, st);
    return -1;
}

template <bool AR>
static int dispatch(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                    const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset,
                    const PeerReduce *pr, cudaStream_t st) {
    if (a_dtype == W4_BF16) {
        if (M <= 8)
            return launch_tma_nt<__nv_bfloat16, 1, AR>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs,
                                                       zero_offset, pr, st);
        return launch_tma_nt<__nv_bfloat16, 2, AR>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset,
                                                   pr, st);
    }
    if (M <= 8)
        return launch_tma_nt<__half, 1, AR>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, pr, st);
    return launch_tma_nt<__half, 2, AR>(a, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, pr, st);
}

// Returns W4_OK, a W4 error, or -1 when the tensor maps cannot be encoded (the
// caller then uses the register-batched kernel).
int gptq_gemv_tma(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                  const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset,
                  cudaStream_t st) {
    return dispatch<false>(a, a_dtype, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, nullptr, st);
}

int gptq_gemv_tma_ar(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                     const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset,
                     const PeerReduce &pr, cudaStream_t st) {
    if (M > 16 || pr.nranks < 2 || pr.nranks > kPeerMaxRanks) return -1;
    return dispatch<true>(a, a_dtype, qweight, qzeros, scales, c, c_dtype, M, N, K, gs, zero_offset, &pr, st);
}

int take_tp_fused_wait_status() {
    unsigned int v = 0;
    W4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_tpf_timeout, sizeof(v)));
    if (v) {
        const unsigned int zero = 0;
        W4_CUDA_TRY(cudaMemcpyToSymbol(g_tpf_timeout, &zero, sizeof(zero)));
        set_error("a peer's tile never arrived in the fused row-parallel all-reduce within the time limit");
        return W4_ERR_TIMEOUT;
    }
    return W4_OK;
}

int take_wait_status() {
    unsigned int v = 0;
    W4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_wait_timeout, sizeof(v)));
    if (v) {
        const unsigned int zero = 0;
        W4_CUDA_TRY(cudaMemcpyToSymbol(g_wait_timeout, &zero, sizeof(zero)));
        set_error("a device-side wait expired (bounded wait in a libw4 kernel)");
        return W4_ERR_TIMEOUT;
    }
    return W4_OK;
}

}  // namespace w4
