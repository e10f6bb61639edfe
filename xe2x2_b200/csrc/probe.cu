// probe.cu -- w4_read_probe: the read bandwidth one kernel launch of a given size attains.
//
// A decode GEMM reads its operands once, so no single launch of it can stream them faster
// than a kernel that does nothing but read the same number of bytes.  This kernel is that
// reference point: every thread streams 16-byte non-coherent loads over its CTA's contiguous
// chunk at full occupancy (four 512-thread CTAs per SM) and folds them into an XOR that is
// stored only if it equals a sentinel, so the loads cannot be elided.  Timed back to back in
// a CUDA graph over buffers larger than L2 it includes the same launch ramp and tail a GEMM
// launch pays, which a long-running copy loop amortises away.
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {
namespace {

constexpr int kProbeThreads = 512;
constexpr int kProbeCtasPerSm = 4;

__global__ void __launch_bounds__(kProbeThreads) read_probe_kernel(const uint4 *__restrict__ p, size_t n16,
                                                                   size_t per_cta, unsigned int *sink) {
    const size_t b = (size_t)blockIdx.x * per_cta;
    const size_t e = b + per_cta < n16 ? b + per_cta : n16;
    unsigned int acc = 0;
#pragma unroll 8
    for (size_t i = b + threadIdx.x; i < e; i += kProbeThreads) {
        const uint4 v = __ldg(p + i);
        acc ^= v.x ^ v.y ^ v.z ^ v.w;
    }
    if (acc == 0x9E3779B9u) sink[0] = acc;  // practically never taken; keeps the loads
}

}  // namespace
}  // namespace w4

extern "C" int w4_read_probe(const void *buf, size_t bytes, unsigned int *sink, void *stream) {
    W4_REQUIRE(buf && sink, W4_ERR_INVALID, "buf and sink are required");
    W4_REQUIRE(bytes > 0 && bytes % 16 == 0, W4_ERR_INVALID, "bytes (%zu) must be a positive multiple of 16", bytes);
    W4_REQUIRE(w4::aligned(buf, 16), W4_ERR_INVALID, "buf must be 16-byte aligned");
    const size_t n16 = bytes / 16;
    const int ctas = w4::kProbeCtasPerSm * w4::num_sms();
    const size_t per = (n16 + ctas - 1) / ctas;
    w4::read_probe_kernel<<<ctas, w4::kProbeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4 *>(buf), n16, per, sink);
    W4_LAUNCH_CHECK();
    return W4_OK;
}
