// tma_util.cuh -- tensor-memory-accelerator copies, mbarriers and tensor-map
// encoding shared by the libw4 kernels (sm_100a).  No copy here uses
// multicast.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <utility>

#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

// Every device-side wait on an mbarrier gives up after this long, so a kernel
// whose copies never land ends with an error status instead of hanging.
constexpr unsigned long long kWaitLimitNs = 200ull * 1000 * 1000;  // 200 ms

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// try_wait that lets the hardware suspend the thread for up to kSuspendNs while the phase
// is incomplete (it resumes as soon as the phase completes), so a waiting warp issues few
// instructions and leaves the issue slots to the warps that compute.
constexpr uint32_t kSuspendNs = 20000;
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return done != 0;
}
// Wait for the phase with the given parity; false if kWaitLimitNs passed first.  The clock is
// read once per 16 suspending tries.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    const uint32_t b = smem_u32(bar);
    if (mbar_try_wait(b, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 16; ++i)
            if (mbar_try_wait_suspend(b, parity)) return true;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
// Untiled bulk copy global -> this CTA's shared memory (no multicast): 16-byte
// aligned addresses, a size that is a multiple of 16, completion on bar.
__device__ __forceinline__ void bulk_load_1d(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Programmatic dependent launch: let the next grid on the stream start its
// prologue now / wait until every grid this one depends on has completed and
// its memory is visible (no-ops when the launch carries no such dependency).
// Fetch a tensor map into the TMA unit's descriptor cache ahead of its first copy.
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// atomicInc with acquire-release semantics at device scope: the writes ordered before it (by
// program order or a CTA barrier) are published with the count, and the writes other threads
// published with their counts are visible after it.
__device__ __forceinline__ unsigned int atom_inc_acq_rel(unsigned int *p, unsigned int limit) {
    unsigned int old;
    asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(limit) : "memory");
    return old;
}
// Row maxima of a decode GEMM's output tile: each value folds |v| into the CTA's shared row
// maxima (fp32 bits compare like the non-negative floats they are), then after the consumers'
// barrier one thread per row folds the CTA's maximum into the global one.
__device__ __forceinline__ void fold_rowmax(unsigned int *rmax, int r, float v) {
    atomicMax(&rmax[r], __float_as_uint(fabsf(v)));
}
template <int CW>
__device__ __forceinline__ void publish_rowmax(const unsigned int *rmax, unsigned int *rowmax, int rows) {
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
    if ((int)threadIdx.x < rows) atomicMax(&rowmax[threadIdx.x], rmax[threadIdx.x]);
}
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Thread-block clusters: a full barrier over every thread of every CTA of the
// cluster (release / acquire at cluster scope), this CTA's rank in it, and a
// load from the same shared-memory offset in another CTA of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ float ld_cluster_f32(const float *p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}


// ---- host: cuTensorMapEncodeTiled through the runtime's driver entry point ----
inline PFN_cuTensorMapEncodeTiled encode_fn() {
    static std::mutex mu;
    static PFN_cuTensorMapEncodeTiled fn = nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
    }
    return fn;
}

// Launch of a decode kernel, with programmatic stream serialisation unless the
// overlap mode is W4_OVERLAP_OFF: the kernel may then start while the previous
// kernel on the stream drains, and orders itself behind it with grid_dep_wait().
// cluster_z > 1: thread-block clusters of (1, 1, cluster_z) CTAs along grid z.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_decode(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 unsigned cluster_z, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    unsigned n = 0;
    if (launch_overlap() != W4_OVERLAP_OFF) {
        at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster_z > 1) {
        at[n].id = cudaLaunchAttributeClusterDimension;
        at[n].val.clusterDim.x = 1;
        at[n].val.clusterDim.y = 1;
        at[n].val.clusterDim.z = cluster_z;
        ++n;
    }
    cfg.attrs = at;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// 3-D tiled map of [d2][d1][d0] elements (d0 innermost; byte strides s1 of d1 and s2 of d2), box
// {b0, b1, 1}: the decode GEMMs read stacked per-expert matrices with the expert as z.
inline bool make_map_3d(CUtensorMap *map, CUtensorMapDataType dt, const void *ptr, uint64_t d0, uint64_t d1,
                        uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle swz) {
    PFN_cuTensorMapEncodeTiled fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {s1, s2};
    const cuuint32_t box[3] = {b0, b1, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, dt, 3, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The token rows of a decode GEMM call as expert groups: expert e owns rows [row0[e], row0[e+1])
// of A and C and token blocks [blk0[e], blk0[e+1]) of grid x.  One group for a plain GEMM.
struct ExpertRows {
    int n;
    int blk0[kMaxExperts + 1];
    int row0[kMaxExperts + 1];
};
__device__ __forceinline__ int expert_of_block(const ExpertRows &g, int b) {
    int e = 0;
    while (e + 1 < g.n && g.blk0[e + 1] <= b) ++e;
    return e;
}
// Host: the table for experts with row offsets off[0..n] (off[0] = 0, nondecreasing) and token
// blocks of `per` rows; false if n is out of range.
inline bool expert_rows(ExpertRows &g, const int *off, int n, int per) {
    if (n < 1 || n > kMaxExperts) return false;
    g.n = n;
    g.blk0[0] = 0;
    for (int e = 0; e <= n; ++e) g.row0[e] = off[e];
    for (int e = 0; e < n; ++e) g.blk0[e + 1] = g.blk0[e] + (off[e + 1] - off[e] + per - 1) / per;
    return true;
}

inline bool make_map_2d(CUtensorMap *map, CUtensorMapDataType dt, const void *ptr, uint64_t d0, uint64_t d1,
                        uint64_t row_bytes, uint32_t b0, uint32_t b1, CUtensorMapSwizzle swz) {
    PFN_cuTensorMapEncodeTiled fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


// Activations as a 3-D tensor [K/64][M][64] (innermost first: 64 k, M tokens,
// K/64 line groups), so one box of {64, rows, KC} lands as KC x rows 128-byte
// lines, each swizzled by its line index.
inline bool make_act_map(CUtensorMap *map, CUtensorMapDataType dt, const void *a, int M, int K, int rows, int kc) {
    PFN_cuTensorMapEncodeTiled fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {64, (cuuint64_t)M, (cuuint64_t)(K / 64)};
    const cuuint64_t strides[2] = {(cuuint64_t)K * 2, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)rows, (cuuint32_t)kc};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, dt, 3, const_cast<void *>(a), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

}  // namespace w4
