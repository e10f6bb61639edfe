// noalloc.cu -- a GPTQ GEMM with the fp8-E4M3 row-scaled output for callers that
// cannot allocate device memory.
//
// w4_gptq_gemm with c_dtype == W4_E4M3 needs scratch: the f32 [M, N] product is
// written first, then every row is scaled by its own absmax and cast.  Usually
// the caller passes that scratch as `workspace`.  Some callers cannot: a host
// binding that only forwards pointers it was handed and has no device
// allocator of its own, or a serving runtime that reserved all of HBM up front
// and forbids any further cudaMalloc.  For them this file holds the scratch in
// a fixed static device array, created when the library is loaded on a device
// and kept until the process exits (kNoAllocMaxElems f32 = 4 MiB per device).
//
// The array's name is only a host-side stand-in for device memory; its real
// device address is looked up once per device with cudaGetSymbolAddress (on
// the first call made with that device current) and cached for the life of the
// process; after cudaDeviceReset the cached address is stale, so do not call
// this again on a device that was reset.  Make the first call before any stream
// capture.  Every call shares the one array, so calls
// that overlap on the GPU (different streams, or threads) race on it: order
// them.  The GEMM overwrites all M*N scratch elements before the cast reads
// them, so nothing has to be cleared between calls.
#include <mutex>

#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

constexpr size_t kNoAllocMaxElems = size_t(1) << 20;  // M * N limit (4 MiB of f32)

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocMaxElems];

static int noalloc_scratch(float **out) {
    static std::mutex mu;
    static float *cache[128] = {};
    int dev = 0;
    W4_CUDA_TRY(cudaGetDevice(&dev));
    W4_REQUIRE(dev >= 0 && dev < 128, W4_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!cache[dev]) {
        void *p = nullptr;
        W4_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        cache[dev] = static_cast<float *>(p);
    }
    *out = cache[dev];
    return W4_OK;
}

}  // namespace w4

extern "C" int w4_gptq_gemm_fp8_noalloc(const void *a, int a_dtype, const int32_t *qweight,
                                        const int32_t *qzeros, const uint16_t *scales,
                                        uint8_t *q_out, float *row_scale, int M, int N, int K,
                                        int group_size, int zero_offset, void *stream) {
    w4::set_error("");
    W4_REQUIRE(a && qweight && scales && q_out && row_scale, W4_ERR_INVALID,
               "a, qweight, scales, q_out and row_scale are required");
    W4_REQUIRE(M >= 1 && N > 0 && K > 0, W4_ERR_INVALID, "M=%d N=%d K=%d", M, N, K);
    W4_REQUIRE(a_dtype == W4_F16 || a_dtype == W4_BF16, W4_ERR_INVALID, "a_dtype must be f16 or bf16");
    W4_REQUIRE(group_size > 0 && K % group_size == 0, W4_ERR_INVALID,
               "K=%d must be a multiple of group_size=%d", K, group_size);
    W4_REQUIRE(K % 32 == 0 && N % 32 == 0 && group_size % 32 == 0, W4_ERR_UNSUPPORTED,
               "need K %% 32 == 0, N %% 32 == 0, group_size %% 32 == 0 (K=%d N=%d gs=%d)", K, N,
               group_size);
    W4_REQUIRE((size_t)M * (size_t)N <= w4::kNoAllocMaxElems, W4_ERR_UNSUPPORTED,
               "M*N = %zu exceeds the static scratch of %zu f32 elements (4 MiB); use "
               "w4_gptq_gemm with a caller workspace",
               (size_t)M * (size_t)N, w4::kNoAllocMaxElems);
    W4_REQUIRE(w4::aligned(a, 16) && w4::aligned(qweight, 16) && w4::aligned(scales, 8),
               W4_ERR_INVALID, "a and qweight must be 16-byte aligned, scales 8-byte aligned");
    W4_REQUIRE((size_t)(K / 8) * (size_t)N < (size_t(1) << 31), W4_ERR_UNSUPPORTED,
               "qweight of %d x %d words exceeds 2^31 elements", K / 8, N);
    float *y = nullptr;
    int rc = w4::noalloc_scratch(&y);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    rc = w4::gptq_gemv(a, a_dtype, qweight, qzeros, scales, y, W4_F32, M, N, K, group_size,
                       zero_offset, nullptr, nullptr, 0, st);  // no scratch for split-K: unsplit
    if (rc) return rc;
    return w4::rowscale_fp8(y, W4_F32, q_out, row_scale, M, N, st);
}
