// w4_api.cu -- the extern "C" boundary of libw4 (include/w4.h).
//
// Every entry point validates its arguments on the host, then enqueues on the
// caller's stream.  Nothing here allocates: scratch comes from the caller's
// workspace, sized by the *_workspace_bytes() functions.
#include <atomic>
#include <mutex>
#include <vector>

#include "w4_common.cuh"
#include "w4_internal.h"
#include "tp_internal.h"

namespace w4 {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

const char *last_error() { return g_err; }

int num_sms() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lk(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

static std::atomic<int> g_overlap{W4_OVERLAP_DEPENDENT};
int launch_overlap() { return g_overlap.load(std::memory_order_relaxed); }

static std::atomic<unsigned long long> g_decode_fallbacks{0};
void note_decode_fallback() { g_decode_fallbacks.fetch_add(1, std::memory_order_relaxed); }

int nvfp4_kn_to_nk(const uint8_t *in, int K, int N, uint8_t *out, cudaStream_t st);

}  // namespace w4

using w4::aligned;

static inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }
static inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

extern "C" {

int w4_abi_version(void) { return W4_ABI_VERSION; }

int w4_set_launch_overlap(int mode) {
    W4_REQUIRE(mode == W4_OVERLAP_OFF || mode == W4_OVERLAP_DEPENDENT || mode == W4_OVERLAP_STATIC_WEIGHTS,
               W4_ERR_INVALID, "overlap mode %d is not one of W4_OVERLAP_*", mode);
    w4::g_overlap.store(mode, std::memory_order_relaxed);
    return W4_OK;
}

int w4_get_launch_overlap(void) { return w4::launch_overlap(); }

unsigned long long w4_decode_fallback_count(void) {
    return w4::g_decode_fallbacks.load(std::memory_order_relaxed);
}

const char *w4_status_string(int status) {
    switch (status) {
        case W4_OK: return "ok";
        case W4_ERR_INVALID: return "invalid argument";
        case W4_ERR_UNSUPPORTED: return "unsupported shape or option";
        case W4_ERR_CUDA: return "CUDA error";
        case W4_ERR_TIMEOUT: return "timed out";
        case W4_ERR_NCCL: return "NCCL error";
        default: return "unknown status";
    }
}

const char *w4_last_error(void) { return w4::last_error(); }

int w4_check_device_status(void) {
    w4::set_error("");
    const int r1 = w4::take_wait_status();
    const int r2 = w4::take_prefill_wait_status();
    const int r3 = w4::take_fp4d_wait_status();
    const int r4 = w4::take_fp4_prefill_wait_status();
    const int r5 = w4::take_tp_wait_status();
    const int r6 = w4::take_tp_fused_wait_status();
    const int r7 = w4::take_rn_wait_status();
    const int r8 = w4::take_decode_wait_status();
    return r1 ? r1 : r2 ? r2 : r3 ? r3 : r4 ? r4 : r5 ? r5 : r6 ? r6 : r7 ? r7 : r8;
}

// ------------------------------------------------------------------ GPTQ
static int check_gptq_common(const int32_t *qweight, const uint16_t *scales, int K, int N,
                             int group_size) {
    W4_REQUIRE(qweight && scales, W4_ERR_INVALID, "qweight and scales are required");
    W4_REQUIRE(K > 0 && N > 0, W4_ERR_INVALID, "K=%d N=%d must be positive", K, N);
    W4_REQUIRE(group_size > 0 && K % group_size == 0, W4_ERR_INVALID,
               "K=%d must be a multiple of group_size=%d", K, group_size);
    W4_REQUIRE(K % 8 == 0 && N % 8 == 0, W4_ERR_INVALID, "K=%d and N=%d must be multiples of 8", K, N);
    return W4_OK;
}

int w4_gptq_dequant(const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                    const int32_t *g_idx, int K, int N, int group_size, int zero_offset,
                    float *w, void *stream) {
    w4::set_error("");
    int rc = check_gptq_common(qweight, scales, K, N, group_size);
    if (rc) return rc;
    W4_REQUIRE(w, W4_ERR_INVALID, "output w is required");
    return w4::gptq_dequant(qweight, qzeros, scales, g_idx, K, N, group_size, zero_offset, w, S(stream));
}

int w4_gptq_repack_act_order(const int32_t *qweight, const int32_t *g_idx, int K, int N,
                             int group_size, int32_t *qweight_out, int32_t *perm_out,
                             void *stream) {
    w4::set_error("");
    W4_REQUIRE(qweight && g_idx && qweight_out && perm_out, W4_ERR_INVALID,
               "qweight, g_idx, qweight_out and perm_out are required");
    W4_REQUIRE(qweight != qweight_out, W4_ERR_INVALID, "qweight_out must not alias qweight");
    W4_REQUIRE(K > 0 && N > 0 && K % 8 == 0 && group_size > 0 && K % group_size == 0,
               W4_ERR_INVALID, "bad shape K=%d N=%d group_size=%d", K, N, group_size);
    return w4::gptq_repack_act_order(qweight, g_idx, K, N, group_size, qweight_out, perm_out, S(stream));
}

// Workspace of w4_gptq_gemm: sync area | gathered activations (act_order) | f32 product
// (e4m3 output) | K-split partials (tensor-core GEMM or decode GEMM).
static size_t gptq_split_bytes(int M, int N, int K, int group_size, int c_dtype) {
    const size_t pf = w4::gptq_prefill_split_bytes(M, N, K, group_size, c_dtype == W4_E4M3 ? W4_F32 : c_dtype);
    const size_t dc = w4::gptq_decode_split_bytes(M, N, K, group_size);
    return pf > dc ? pf : dc;
}

size_t w4_gptq_workspace_bytes(int M, int N, int K, int group_size, int has_perm, int c_dtype) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    size_t ws = W4_WORKSPACE_SYNC_BYTES;
    if (has_perm) ws += align256((size_t)M * K * 2);
    if (c_dtype == W4_E4M3) ws += align256((size_t)M * N * 4);
    ws += align256(gptq_split_bytes(M, N, K, group_size, c_dtype));
    return ws;
}

}  // extern "C"

namespace w4 {
// The argument rules of w4_gptq_gemm (everything but the workspace).
int check_gptq_gemm(const void *a, int a_dtype, const int32_t *qweight, const uint16_t *scales, const void *c,
                    int c_dtype, const float *row_scale, int M, int N, int K, int group_size) {
    int rc = check_gptq_common(qweight, scales, K, N, group_size);
    if (rc) return rc;
    W4_REQUIRE(a && c, W4_ERR_INVALID, "a and c are required");
    W4_REQUIRE(M >= 1, W4_ERR_INVALID, "M=%d must be >= 1", M);
    W4_REQUIRE(a_dtype == W4_F16 || a_dtype == W4_BF16, W4_ERR_INVALID, "a_dtype must be f16 or bf16");
    W4_REQUIRE(c_dtype == W4_F16 || c_dtype == W4_BF16 || c_dtype == W4_F32 || c_dtype == W4_E4M3,
               W4_ERR_INVALID, "c_dtype must be f16, bf16, f32 or e4m3");
    W4_REQUIRE(c_dtype != W4_E4M3 || row_scale, W4_ERR_INVALID, "e4m3 output needs row_scale");
    W4_REQUIRE(K % 32 == 0 && N % 32 == 0 && group_size % 32 == 0, W4_ERR_UNSUPPORTED,
               "need K %% 32 == 0, N %% 32 == 0, group_size %% 32 == 0 (K=%d N=%d gs=%d)", K, N,
               group_size);
    W4_REQUIRE(aligned(a, 16) && aligned(qweight, 16) && aligned(scales, 8), W4_ERR_INVALID,
               "a and qweight must be 16-byte aligned, scales 8-byte aligned");
    W4_REQUIRE((size_t)(K / 8) * (size_t)N < (size_t(1) << 31), W4_ERR_UNSUPPORTED,
               "qweight of %d x %d words exceeds 2^31 elements", K / 8, N);
    return W4_OK;
}
}  // namespace w4

extern "C" {

int w4_gptq_gemm(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                 const uint16_t *scales, const int32_t *perm, void *c, int c_dtype,
                 float *row_scale, int M, int N, int K, int group_size, int zero_offset,
                 void *workspace, size_t workspace_bytes, void *stream) {
    w4::set_error("");
    int rc = w4::check_gptq_gemm(a, a_dtype, qweight, scales, c, c_dtype, row_scale, M, N, K, group_size);
    if (rc) return rc;
    const size_t need = w4_gptq_workspace_bytes(M, N, K, group_size, perm != nullptr, c_dtype);
    const size_t split = align256(gptq_split_bytes(M, N, K, group_size, c_dtype));
    // At decode sizes the K-split partials are optional: without them the GEMM runs unsplit.
    const size_t least = M <= 16 ? need - split : need;
    W4_REQUIRE(workspace_bytes >= least && workspace && aligned(workspace, 256), W4_ERR_INVALID,
               "a 256-byte aligned workspace of %zu bytes is needed (%zu given), its first %d bytes zero",
               need, workspace_bytes, W4_WORKSPACE_SYNC_BYTES);
    cudaStream_t st = S(stream);
    char *sync = static_cast<char *>(workspace);
    char *ws = sync + W4_WORKSPACE_SYNC_BYTES;
    const void *a_eff = a;
    if (perm) {
        uint16_t *ap = reinterpret_cast<uint16_t *>(ws);
        ws += align256((size_t)M * K * 2);
        rc = w4::gather_cols(static_cast<const uint16_t *>(a), perm, M, K, ap, st);
        if (rc) return rc;
        a_eff = ap;
    }
    void *out = c;
    if (c_dtype == W4_E4M3) {
        out = ws;
        ws += align256((size_t)M * N * 4);
    }
    const size_t have = workspace_bytes - (size_t)(ws - sync);
    if (c_dtype == W4_E4M3 && M <= 16 && N % 8 == 0 && aligned(c, 8) && !w4::prefer_register_gemv(M, N, K)) {
        // decode: the GEMM folds the row maxima of its f32 product into the sync area, so the
        // cast reads the product once
        unsigned int *sw = reinterpret_cast<unsigned int *>(sync);
        rc = w4::gptq_gemv_decode(a_eff, a_dtype, qweight, qzeros, scales, out, W4_F32, M, N, K, group_size,
                                  zero_offset, sync, split ? ws : nullptr, split < have ? split : have,
                                  sw + w4::kSyncRowMax, st);
        if (rc == W4_OK)
            return w4::rowscale_fp8_amax(static_cast<const float *>(out), sw + w4::kSyncRowMax, sw + w4::kSyncRowCnt,
                                         static_cast<uint8_t *>(c), row_scale, M, N, st);
        if (rc != -1) return rc;
    }
    rc = w4::gptq_gemv(a_eff, a_dtype, qweight, qzeros, scales, out, c_dtype == W4_E4M3 ? W4_F32 : c_dtype, M, N,
                       K, group_size, zero_offset, sync, split ? ws : nullptr, split < have ? split : have, st);
    if (rc || c_dtype != W4_E4M3) return rc;
    return w4::rowscale_fp8(static_cast<const float *>(out), W4_F32, static_cast<uint8_t *>(c), row_scale, M, N, st);
}

// ------------------------------------------------------------------ grouped (MoE)
static int check_offsets(const int32_t *off, int n, int *rows) {
    W4_REQUIRE(off && n >= 1 && n <= w4::kMaxExperts, W4_ERR_INVALID, "offsets and 1..%d experts are required",
               w4::kMaxExperts);
    W4_REQUIRE(off[0] == 0, W4_ERR_INVALID, "offsets[0] must be 0");
    for (int e = 0; e < n; ++e)
        W4_REQUIRE(off[e + 1] >= off[e], W4_ERR_INVALID, "offsets must be nondecreasing (expert %d)", e);
    *rows = off[n];
    return W4_OK;
}

// Rows of the largest expert (offsets already checked).
static int max_expert_rows(const int32_t *off, int n) {
    int m = 0;
    for (int e = 0; e < n; ++e) m = off[e + 1] - off[e] > m ? off[e + 1] - off[e] : m;
    return m;
}

size_t w4_gptq_gemm_grouped_workspace_bytes(const int32_t *offsets, int num_experts, int N, int K, int group_size,
                                            int c_dtype) {
    int rows = 0;
    if (check_offsets(offsets, num_experts, &rows) || N <= 0 || K <= 0 || group_size <= 0) return 0;
    size_t ws = W4_WORKSPACE_SYNC_BYTES;
    if (c_dtype == W4_E4M3) ws += align256((size_t)rows * N * 4);
    const int odt = c_dtype == W4_E4M3 ? W4_F32 : c_dtype;
    const size_t dec = w4::gptq_decode_grouped_split_bytes(offsets, num_experts, N, K, group_size);
    const size_t pf = max_expert_rows(offsets, num_experts) >= w4::kGroupedPrefillMinRows
                          ? w4::gptq_prefill_grouped_split_bytes(offsets, num_experts, N, K, group_size, odt)
                          : 0;
    return ws + align256(dec > pf ? dec : pf);
}

int w4_gptq_gemm_grouped(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                         const uint16_t *scales, const int32_t *offsets, int num_experts, void *c, int c_dtype,
                         float *row_scale, int N, int K, int group_size, int zero_offset, void *workspace,
                         size_t workspace_bytes, void *stream) {
    w4::set_error("");
    int rows = 0;
    int rc = check_offsets(offsets, num_experts, &rows);
    if (rc) return rc;
    rc = w4::check_gptq_gemm(a, a_dtype, qweight, scales, c, c_dtype, row_scale, rows > 0 ? rows : 1, N, K,
                             group_size);
    if (rc) return rc;
    const size_t need = w4_gptq_gemm_grouped_workspace_bytes(offsets, num_experts, N, K, group_size, c_dtype);
    W4_REQUIRE(workspace_bytes >= need && workspace && aligned(workspace, 256), W4_ERR_INVALID,
               "a 256-byte aligned workspace of %zu bytes is needed (%zu given), its first %d bytes zero", need,
               workspace_bytes, W4_WORKSPACE_SYNC_BYTES);
    if (rows == 0) return W4_OK;
    cudaStream_t st = S(stream);
    char *sync = static_cast<char *>(workspace);
    char *ws = sync + W4_WORKSPACE_SYNC_BYTES;
    void *out = c;
    if (c_dtype == W4_E4M3) {
        out = ws;
        ws += align256((size_t)rows * N * 4);
    }
    const int odt = c_dtype == W4_E4M3 ? W4_F32 : c_dtype;
    const size_t have = workspace_bytes - (size_t)(ws - sync);
    rc = -1;
    if (max_expert_rows(offsets, num_experts) >= w4::kGroupedPrefillMinRows)
        rc = w4::gptq_prefill_grouped(a, a_dtype, qweight, qzeros, scales, offsets, num_experts, out, odt, N, K,
                                      group_size, zero_offset, ws, have, st);
    if (rc == -1)
        rc = w4::gptq_gemv_decode_grouped(a, a_dtype, qweight, qzeros, scales, offsets, num_experts, out, odt, N, K,
                                          group_size, zero_offset, sync, ws, have, st);
    if (rc == -1) {
        w4::set_error("grouped GPTQ GEMM: shape not handled (N %% 32, K %% 8, group size 32, 64 or a multiple of "
                      "128, 16-byte aligned tensors)");
        return W4_ERR_UNSUPPORTED;
    }
    if (rc || c_dtype != W4_E4M3) return rc;
    return w4::rowscale_fp8(out, W4_F32, static_cast<uint8_t *>(c), row_scale, rows, N, st);
}

size_t w4_nvfp4_gemm_grouped_workspace_bytes(const int32_t *offsets, int num_experts, int N, int K, int c_dtype) {
    int rows = 0;
    if (check_offsets(offsets, num_experts, &rows) || N <= 0 || K <= 0) return 0;
    size_t ws = W4_WORKSPACE_SYNC_BYTES;
    if (c_dtype == W4_E4M3) ws += align256((size_t)rows * N * 4);
    const int odt = c_dtype == W4_E4M3 ? W4_F32 : c_dtype;
    const size_t dec = w4::nvfp4_decode_grouped_split_bytes(offsets, num_experts, N, K);
    const size_t pf = max_expert_rows(offsets, num_experts) >= w4::kGroupedPrefillMinRows
                          ? w4::nvfp4_w4a16_prefill_grouped_split_bytes(offsets, num_experts, N, K, odt)
                          : 0;
    return ws + align256(dec > pf ? dec : pf);
}

int w4_nvfp4_gemm_grouped(const void *a, const uint8_t *w, const uint8_t *scale, const float *global_scale,
                          const int32_t *offsets, int num_experts, void *c, int c_dtype, float *row_scale, int N, int K,
                          void *workspace, size_t workspace_bytes, void *stream) {
    w4::set_error("");
    int rows = 0;
    int rc = check_offsets(offsets, num_experts, &rows);
    if (rc) return rc;
    W4_REQUIRE(a && w && scale && global_scale && c, W4_ERR_INVALID, "a, w, scale, global_scale and c are required");
    W4_REQUIRE(N > 0 && K > 0 && N % 32 == 0 && K % 64 == 0, W4_ERR_UNSUPPORTED,
               "need N %% 32 == 0 and K %% 64 == 0 (N=%d K=%d)", N, K);
    W4_REQUIRE(c_dtype == W4_F16 || c_dtype == W4_BF16 || c_dtype == W4_F32 || c_dtype == W4_E4M3, W4_ERR_INVALID,
               "c_dtype must be f16, bf16, f32 or e4m3");
    W4_REQUIRE(c_dtype != W4_E4M3 || row_scale, W4_ERR_INVALID, "e4m3 output needs row_scale");
    W4_REQUIRE(aligned(a, 16) && aligned(w, 16) && aligned(scale, 16), W4_ERR_INVALID,
               "a, w and scale must be 16-byte aligned");
    const size_t need = w4_nvfp4_gemm_grouped_workspace_bytes(offsets, num_experts, N, K, c_dtype);
    W4_REQUIRE(workspace_bytes >= need && workspace && aligned(workspace, 256), W4_ERR_INVALID,
               "a 256-byte aligned workspace of %zu bytes is needed (%zu given), its first %d bytes zero", need,
               workspace_bytes, W4_WORKSPACE_SYNC_BYTES);
    if (rows == 0) return W4_OK;
    cudaStream_t st = S(stream);
    char *sync = static_cast<char *>(workspace);
    char *ws = sync + W4_WORKSPACE_SYNC_BYTES;
    void *out = c;
    if (c_dtype == W4_E4M3) {
        out = ws;
        ws += align256((size_t)rows * N * 4);
    }
    const int odt = c_dtype == W4_E4M3 ? W4_F32 : c_dtype;
    const size_t have = workspace_bytes - (size_t)(ws - sync);
    rc = -1;
    if (max_expert_rows(offsets, num_experts) >= w4::kGroupedPrefillMinRows)
        rc = w4::nvfp4_w4a16_prefill_grouped(static_cast<const uint16_t *>(a), w, scale, global_scale, offsets,
                                             num_experts, out, odt, N, K, ws, have, st);
    if (rc == -1)
        rc = w4::nvfp4_gemv_decode_grouped(static_cast<const uint16_t *>(a), w, scale, W4_E4M3, global_scale,
                                           offsets, num_experts, out, odt, N, K, sync, ws, have, st);
    if (rc == -1) {
        w4::set_error("grouped NVFP4 GEMM: shape not handled by the decode kernel");
        return W4_ERR_UNSUPPORTED;
    }
    if (rc || c_dtype != W4_E4M3) return rc;
    return w4::rowscale_fp8(out, W4_F32, static_cast<uint8_t *>(c), row_scale, rows, N, st);
}

int w4_gptq_gemm_s4a(const uint8_t *a_s4, const uint8_t *b_s4, const float *a_scale,
                     const uint16_t *b_scale, uint16_t *c, int rows, int cols, int dk,
                     void *stream) {
    w4::set_error("");
    W4_REQUIRE(a_s4 && b_s4 && a_scale && b_scale && c, W4_ERR_INVALID, "null pointer argument");
    W4_REQUIRE(rows >= 1 && cols >= 1 && dk >= 128 && dk % 128 == 0, W4_ERR_INVALID,
               "shape rows=%d cols=%d dk=%d (dk must be a multiple of 128)", rows, cols, dk);
    return w4::gptq_s4a(a_s4, b_s4, a_scale, b_scale, c, rows, cols, dk, S(stream));
}

// ------------------------------------------------------------------ NVFP4
static int check_nvfp4_w(const uint8_t *w, int layout, const void *scale, int scale_dtype,
                         const float *global_scale, int K, int N) {
    W4_REQUIRE(w && scale, W4_ERR_INVALID, "w and scale are required");
    W4_REQUIRE(layout == W4_NVFP4_KN || layout == W4_NVFP4_NK, W4_ERR_INVALID, "bad layout %d", layout);
    W4_REQUIRE(scale_dtype == W4_E4M3 || scale_dtype == W4_BF16 || scale_dtype == W4_E4M3_ATOMS, W4_ERR_INVALID,
               "scale_dtype must be e4m3, e4m3 atoms or bf16");
    W4_REQUIRE(scale_dtype == W4_BF16 || global_scale, W4_ERR_INVALID,
               "e4m3 block scales need the fp32 tensor scale");
    W4_REQUIRE(scale_dtype != W4_BF16 || !global_scale, W4_ERR_INVALID,
               "bf16 (folded) block scales take no tensor scale");
    W4_REQUIRE(K > 0 && N > 0 && K % 16 == 0, W4_ERR_INVALID, "K=%d must be a positive multiple of 16", K);
    return W4_OK;
}

int w4_nvfp4_dequant(const uint8_t *w, int layout, const void *scale, int scale_dtype,
                     const float *global_scale, int K, int N, float *out, void *stream) {
    w4::set_error("");
    int rc = check_nvfp4_w(w, layout, scale, scale_dtype, global_scale, K, N);
    if (rc) return rc;
    W4_REQUIRE(scale_dtype != W4_E4M3_ATOMS, W4_ERR_UNSUPPORTED, "dequant reads [K/16, N] block scales");
    W4_REQUIRE(out, W4_ERR_INVALID, "out is required");
    return w4::nvfp4_dequant(w, layout, scale, scale_dtype, global_scale, K, N, out, S(stream));
}

int w4_nvfp4_quant_act(const uint16_t *a, int M, int K, const float *a_global, uint8_t *codes,
                       uint8_t *sf, void *stream) {
    w4::set_error("");
    W4_REQUIRE(a && a_global && codes && sf, W4_ERR_INVALID, "null pointer argument");
    W4_REQUIRE(M >= 1 && K > 0 && K % 16 == 0, W4_ERR_INVALID, "M=%d K=%d (K %% 16 == 0)", M, K);
    W4_REQUIRE(aligned(a, 16) && aligned(codes, 8), W4_ERR_INVALID, "a 16-byte, codes 8-byte aligned");
    return w4::nvfp4_quant_act(a, M, K, a_global, codes, sf, S(stream));
}

size_t w4_nvfp4_workspace_bytes(int M, int N, int K, int act_mode, int c_dtype) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    size_t ws = W4_WORKSPACE_SYNC_BYTES;
    if (act_mode == W4_ACT_NVFP4) ws += w4::nvfp4_prefill_workspace(M, N, K);
    if (c_dtype == W4_E4M3) ws += align256((size_t)M * N * 4);
    // split-K partials of the W4A16 tensor-core GEMM or of the decode GEMM, whichever the shape
    // takes (after the f32 product when the output is e4m3)
    if (act_mode == W4_ACT_W4A16) {
        const size_t pf = w4::nvfp4_w4a16_prefill_split_bytes(M, N, K, c_dtype == W4_E4M3 ? W4_F32 : c_dtype);
        const size_t dec = w4::nvfp4_decode_split_bytes(M, N, K);
        ws += align256(pf > dec ? pf : dec);
    }
    return ws;
}

int w4_nvfp4_gemm(const void *a, const uint8_t *w, int layout, const void *scale,
                  int scale_dtype, const float *global_scale, int act_mode,
                  const float *a_global, void *c, int c_dtype, float *row_scale, int M, int N,
                  int K, void *workspace, size_t workspace_bytes, void *stream) {
    w4::set_error("");
    int rc = check_nvfp4_w(w, layout, scale, scale_dtype, global_scale, K, N);
    if (rc) return rc;
    W4_REQUIRE(a && c, W4_ERR_INVALID, "a and c are required");
    W4_REQUIRE(M >= 1, W4_ERR_INVALID, "M=%d must be >= 1", M);
    W4_REQUIRE(act_mode == W4_ACT_W4A16 || act_mode == W4_ACT_NVFP4, W4_ERR_INVALID, "bad act_mode");
    W4_REQUIRE(act_mode != W4_ACT_NVFP4 || a_global, W4_ERR_INVALID, "NVFP4 activations need a_global");
    W4_REQUIRE(c_dtype == W4_F16 || c_dtype == W4_BF16 || c_dtype == W4_F32 || c_dtype == W4_E4M3,
               W4_ERR_INVALID, "c_dtype must be f16, bf16, f32 or e4m3");
    W4_REQUIRE(c_dtype != W4_E4M3 || row_scale, W4_ERR_INVALID, "e4m3 output needs row_scale");
    W4_REQUIRE(layout == W4_NVFP4_NK, W4_ERR_UNSUPPORTED,
               "the GEMM reads the K-contiguous [N, K/2] layout; transpose [K/2, N] weights once "
               "with w4_nvfp4_repack_kn_to_nk");
    W4_REQUIRE(K % 128 == 0 && N % 32 == 0, W4_ERR_UNSUPPORTED,
               "need K %% 128 == 0 and N %% 32 == 0 (K=%d N=%d)", K, N);
    W4_REQUIRE(scale_dtype != W4_E4M3_ATOMS || act_mode == W4_ACT_NVFP4, W4_ERR_UNSUPPORTED,
               "rearranged scale atoms are read by the NVFP4-activation GEMM only");
    W4_REQUIRE(aligned(a, 16) && aligned(w, 16), W4_ERR_INVALID, "a and w must be 16-byte aligned");
    const size_t need = w4_nvfp4_workspace_bytes(M, N, K, act_mode, c_dtype);
    W4_REQUIRE(workspace_bytes >= need && workspace && aligned(workspace, 256), W4_ERR_INVALID,
               "a 256-byte aligned workspace of %zu bytes is needed (%zu given), its first %d bytes zero",
               need, workspace_bytes, W4_WORKSPACE_SYNC_BYTES);
    cudaStream_t st = S(stream);
    char *const wsbase = static_cast<char *>(workspace) + W4_WORKSPACE_SYNC_BYTES;
    if (act_mode == W4_ACT_NVFP4) {
        // block-scaled tensor-core GEMM on NVFP4 activations (nvfp4_prefill.cu)
        W4_REQUIRE(scale_dtype == W4_E4M3 || scale_dtype == W4_E4M3_ATOMS, W4_ERR_UNSUPPORTED,
                   "NVFP4 activations need E4M3 weight block scales (the MMA scales are UE4M3)");
        W4_REQUIRE(K % 256 == 0 && N % 128 == 0, W4_ERR_UNSUPPORTED,
                   "NVFP4 activations need K %% 256 == 0 and N %% 128 == 0 (K=%d N=%d)", K, N);
        char *wsb = wsbase;
        void *out = c;
        int odt = c_dtype;
        if (c_dtype == W4_E4M3) {
            out = wsb;
            odt = W4_F32;
            wsb += align256((size_t)M * N * 4);
        }
        rc = w4::nvfp4_prefill(static_cast<const uint16_t *>(a), a_global, w, static_cast<const uint8_t *>(scale),
                               scale_dtype == W4_E4M3_ATOMS, global_scale, out, odt, M, N, K, wsb, st);
        if (rc < 0) {
            w4::set_error("NVFP4-activation GEMM: tensor maps could not be encoded for this shape");
            return W4_ERR_UNSUPPORTED;
        }
        if (rc || c_dtype != W4_E4M3) return rc;
        return w4::rowscale_fp8(out, W4_F32, static_cast<uint8_t *>(c), row_scale, M, N, st);
    }
    // W4A16: the decode kernels up to 16 tokens where prefer_fp4_decode says so, else the
    // tensor-core GEMM (E4M3 block scales)
    char *wsb = wsbase;
    void *out = c;
    int odt = c_dtype;
    if (c_dtype == W4_E4M3) {
        out = wsb;
        odt = W4_F32;
        wsb += align256((size_t)M * N * 4);
    }
    rc = -1;
    const size_t have = workspace_bytes - (size_t)(wsb - static_cast<char *>(workspace));
    if (c_dtype == W4_E4M3 && w4::prefer_fp4_decode(M, N, K) && N % 8 == 0 && aligned(c, 8)) {
        // decode: the GEMM folds the row maxima of its f32 product into the sync area, so the
        // cast reads the product once
        unsigned int *sw = static_cast<unsigned int *>(workspace);
        rc = w4::nvfp4_gemv_decode(static_cast<const uint16_t *>(a), w, scale, scale_dtype, global_scale, out, odt,
                                   M, N, K, workspace, wsb, have, sw + w4::kSyncRowMax, st);
        if (rc == W4_OK)
            return w4::rowscale_fp8_amax(static_cast<const float *>(out), sw + w4::kSyncRowMax, sw + w4::kSyncRowCnt,
                                         static_cast<uint8_t *>(c), row_scale, M, N, st);
        if (rc != -1) return rc;
    }
    if (scale_dtype == W4_E4M3) {
        const size_t split = w4::nvfp4_w4a16_prefill_split_bytes(M, N, K, odt);
        rc = w4::nvfp4_w4a16_prefill(static_cast<const uint16_t *>(a), w, static_cast<const uint8_t *>(scale),
                                     global_scale, out, odt, M, N, K, split ? wsb : nullptr, split, st);
    }
    if (rc == -1)
        rc = w4::nvfp4_gemv(static_cast<const uint16_t *>(a), w, layout, scale, scale_dtype, global_scale, out, odt,
                            M, N, K, workspace, wsb, have, st);
    if (rc || c_dtype != W4_E4M3) return rc;
    return w4::rowscale_fp8(out, W4_F32, static_cast<uint8_t *>(c), row_scale, M, N, st);
}

size_t w4_nvfp4_act_codes_bytes(int M, int K) {
    if (M <= 0 || K <= 0 || K % 64) return 0;
    return (size_t)(M + 127) / 128 * 128 * (size_t)(K / 2);
}

int w4_rmsnorm_quant_nvfp4(const void *x, int x_dtype, const void *gamma, float eps, const float *a_global,
                           uint8_t *codes, uint8_t *sf_atoms, int M, int K, void *stream) {
    w4::set_error("");
    W4_REQUIRE(x && a_global && codes && sf_atoms, W4_ERR_INVALID, "null pointer argument");
    W4_REQUIRE(x_dtype == W4_F16 || x_dtype == W4_BF16, W4_ERR_INVALID, "x_dtype must be f16 or bf16");
    W4_REQUIRE(M >= 1 && K > 0 && K % 64 == 0, W4_ERR_INVALID, "M=%d K=%d (K %% 64 == 0)", M, K);
    W4_REQUIRE(eps >= 0.f, W4_ERR_INVALID, "eps must be >= 0");
    W4_REQUIRE(aligned(x, 16) && (!gamma || aligned(gamma, 16)) && aligned(codes, 16), W4_ERR_INVALID,
               "x, gamma and codes must be 16-byte aligned");
    return w4::rmsnorm_nvfp4(x, x_dtype, gamma, eps, a_global, codes, sf_atoms, M, K, S(stream));
}

size_t w4_nvfp4_gemm_q_workspace_bytes(int M, int N, int K, int scale_dtype, int c_dtype) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    size_t ws = W4_WORKSPACE_SYNC_BYTES + w4::nvfp4_prefill_q_workspace(M, N, K, scale_dtype == W4_E4M3);
    if (c_dtype == W4_E4M3) ws += align256((size_t)M * N * 4);
    return ws;
}

int w4_nvfp4_gemm_q(const uint8_t *a_codes, const uint8_t *a_sf_atoms, const float *a_global, const uint8_t *w,
                    int layout, const void *scale, int scale_dtype, const float *global_scale, void *c,
                    int c_dtype, float *row_scale, int M, int N, int K, void *workspace, size_t workspace_bytes,
                    void *stream) {
    w4::set_error("");
    int rc = check_nvfp4_w(w, layout, scale, scale_dtype, global_scale, K, N);
    if (rc) return rc;
    W4_REQUIRE(a_codes && a_sf_atoms && a_global && c, W4_ERR_INVALID,
               "a_codes, a_sf_atoms, a_global and c are required");
    W4_REQUIRE(M >= 1, W4_ERR_INVALID, "M=%d must be >= 1", M);
    W4_REQUIRE(c_dtype == W4_F16 || c_dtype == W4_BF16 || c_dtype == W4_F32 || c_dtype == W4_E4M3,
               W4_ERR_INVALID, "c_dtype must be f16, bf16, f32 or e4m3");
    W4_REQUIRE(c_dtype != W4_E4M3 || row_scale, W4_ERR_INVALID, "e4m3 output needs row_scale");
    W4_REQUIRE(layout == W4_NVFP4_NK, W4_ERR_UNSUPPORTED, "the GEMM reads the K-contiguous [N, K/2] layout");
    W4_REQUIRE(scale_dtype == W4_E4M3 || scale_dtype == W4_E4M3_ATOMS, W4_ERR_UNSUPPORTED,
               "NVFP4 activations need E4M3 weight block scales (the MMA scales are UE4M3)");
    W4_REQUIRE(K % 256 == 0 && N % 128 == 0, W4_ERR_UNSUPPORTED,
               "NVFP4 activations need K %% 256 == 0 and N %% 128 == 0 (K=%d N=%d)", K, N);
    W4_REQUIRE(aligned(a_codes, 16) && aligned(w, 16) && aligned(a_sf_atoms, 16) &&
                   (scale_dtype != W4_E4M3_ATOMS || aligned(scale, 16)),
               W4_ERR_INVALID, "a_codes, a_sf_atoms, w and scale atoms must be 16-byte aligned");
    const size_t need = w4_nvfp4_gemm_q_workspace_bytes(M, N, K, scale_dtype, c_dtype);
    W4_REQUIRE(workspace_bytes >= need && workspace && aligned(workspace, 256), W4_ERR_INVALID,
               "a 256-byte aligned workspace of %zu bytes is needed (%zu given), its first %d bytes zero",
               need, workspace_bytes, W4_WORKSPACE_SYNC_BYTES);
    cudaStream_t st = S(stream);
    char *wsb = static_cast<char *>(workspace) + W4_WORKSPACE_SYNC_BYTES;
    void *out = c;
    int odt = c_dtype;
    if (c_dtype == W4_E4M3) {
        out = wsb;
        odt = W4_F32;
        wsb += align256((size_t)M * N * 4);
    }
    rc = w4::nvfp4_prefill_q(a_codes, a_sf_atoms, a_global, w, static_cast<const uint8_t *>(scale),
                             scale_dtype == W4_E4M3_ATOMS, global_scale, out, odt, M, N, K, wsb, st);
    if (rc < 0) {
        w4::set_error("NVFP4-activation GEMM: tensor maps could not be encoded for this shape");
        return W4_ERR_UNSUPPORTED;
    }
    if (rc || c_dtype != W4_E4M3) return rc;
    return w4::rowscale_fp8(out, W4_F32, static_cast<uint8_t *>(c), row_scale, M, N, st);
}

int w4_nvfp4_repack_kn_to_nk(const uint8_t *w_kn, int K, int N, uint8_t *w_nk, void *stream) {
    w4::set_error("");
    W4_REQUIRE(w_kn && w_nk && w_kn != w_nk, W4_ERR_INVALID, "distinct w_kn and w_nk are required");
    W4_REQUIRE(K > 0 && N > 0 && K % 2 == 0, W4_ERR_INVALID, "K=%d N=%d", K, N);
    return w4::nvfp4_kn_to_nk(w_kn, K, N, w_nk, S(stream));
}

size_t w4_nvfp4_scale_atoms_bytes(int N, int K) {
    if (N <= 0 || K <= 0 || K % 64) return 0;
    return (size_t)(N + 127) / 128 * 128 * (size_t)(K / 16);
}

int w4_nvfp4_repack_scales(const uint8_t *scale, int K, int N, uint8_t *atoms, void *stream) {
    w4::set_error("");
    W4_REQUIRE(scale && atoms && (const void *)scale != (const void *)atoms, W4_ERR_INVALID,
               "distinct scale and atoms buffers are required");
    W4_REQUIRE(K > 0 && N > 0 && K % 64 == 0, W4_ERR_INVALID, "K=%d must be a positive multiple of 64", K);
    return w4::nvfp4_sf_atoms(scale, N, K / 16, 1, N, atoms, S(stream));
}

int w4_nvfp4_lut_gemm_s8a(const int8_t *a, const uint8_t *packed, const float *a_s,
                          const float *b_s, uint16_t *c, int rows, int cols, int dk,
                          void *stream) {
    w4::set_error("");
    W4_REQUIRE(a && packed && a_s && b_s && c, W4_ERR_INVALID, "null pointer argument");
    W4_REQUIRE(rows >= 1 && cols >= 1 && dk >= 2 && dk % 2 == 0, W4_ERR_INVALID,
               "shape rows=%d cols=%d dk=%d", rows, cols, dk);
    return w4::nvfp4_lut_s8a(a, packed, a_s, b_s, c, rows, cols, dk, S(stream));
}

// ------------------------------------------------------------------ epilogue quant
int w4_rmsnorm_quant_s8(const uint16_t *x, int8_t *q, float *scale, int M, int K, float eps,
                        void *stream) {
    w4::set_error("");
    W4_REQUIRE(x && q && scale, W4_ERR_INVALID, "null pointer argument");
    W4_REQUIRE(M >= 1 && K >= 8 && K % 8 == 0, W4_ERR_INVALID, "M=%d K=%d (K %% 8 == 0)", M, K);
    W4_REQUIRE(aligned(x, 16) && aligned(q, 8), W4_ERR_INVALID, "x 16-byte, q 8-byte aligned");
    return w4::rmsnorm_quant_s8(x, q, scale, M, K, eps, S(stream));
}

int w4_rowscale_fp8(const void *y, int y_dtype, uint8_t *q, float *row_scale, int M, int N,
                    void *stream) {
    w4::set_error("");
    W4_REQUIRE(y && q && row_scale, W4_ERR_INVALID, "null pointer argument");
    W4_REQUIRE(M >= 1 && N >= 1, W4_ERR_INVALID, "M=%d N=%d", M, N);
    W4_REQUIRE(y_dtype == W4_F16 || y_dtype == W4_BF16 || y_dtype == W4_F32, W4_ERR_INVALID,
               "y_dtype must be f16, bf16 or f32");
    return w4::rowscale_fp8(y, y_dtype, q, row_scale, M, N, S(stream));
}

}  // extern "C"
