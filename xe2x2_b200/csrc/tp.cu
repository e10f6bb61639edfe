// tp.cu -- tensor-parallel GPTQ linear layers: column / row sharding with an
// NCCL all-reduce of the row-parallel partial outputs.
//
// The reference's only tensor-parallel piece is the collective itself: an
// in-place bf16 all_reduce(SUM) between two ranks through torch's xccl backend
// (parallel/tp2/bench_xccl_p2p0.py:235-251, parallel/tp2/bench_host_ar.py:91-105).
// Here one process drives one GPU; its communicator is an NCCL communicator
// over NVLink/NVSwitch created from a 128-byte unique id that the ranks
// exchange through whatever bootstrap the host has (torch.distributed's store
// in the Python layer).
//
// NCCL is resolved at run time (dlopen of libnccl.so.2: the copy the process
// already loaded, else the system one), so libw4 loads and its single-GPU
// entry points work on hosts without NCCL; the w4_tp_* calls then return
// W4_ERR_UNSUPPORTED.
//
// Failure handling: the communicator is created non-blocking, and
// w4_tp_comm_init / w4_tp_wait poll with a time limit.  When a peer never
// joins or never reaches the collective, the wait expires, the communicator
// is aborted (NCCL stops its in-flight kernels) and W4_ERR_TIMEOUT is
// returned; the communicator is unusable afterwards.
#include <chrono>
#include <thread>

#include "tp_internal.h"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {
namespace {

#define W4_NCCL_API()                                                                                     \
    const NcclApi &api = nccl();                                                                          \
    W4_REQUIRE(api.ok, W4_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded")

int nccl_fail(const NcclApi &api, ncclResult_t r, const char *what) {
    set_error("%s: NCCL error %d (%s)", what, (int)r, api.error_string(r));
    return W4_ERR_NCCL;
}

using Clock = std::chrono::steady_clock;

// Poll a non-blocking communicator until its pending operation (init) is done.
int wait_comm_ready(const NcclApi &api, w4_tp_comm *c, int timeout_ms) {
    const auto t0 = Clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = api.comm_get_async_error(c->comm, &st);
        if (r != ncclSuccess) return nccl_fail(api, r, "ncclCommGetAsyncError");
        if (st == ncclSuccess) return W4_OK;
        if (st != ncclInProgress) {
            api.comm_abort(c->comm);
            c->dead = true;
            return nccl_fail(api, st, "communicator");
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > timeout_ms) {
            api.comm_abort(c->comm);
            c->dead = true;
            set_error("NCCL communicator not ready after %d ms (a peer did not join); aborted", timeout_ms);
            return W4_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

ncclDataType_t nccl_dtype(int dt) {
    switch (dt) {
    case W4_F16: return ncclFloat16;
    case W4_BF16: return ncclBfloat16;
    default: return ncclFloat32;
    }
}

}  // namespace
}  // namespace w4

using namespace w4;

extern "C" int w4_tp_get_unique_id(uint8_t *id) {
    set_error("");
    W4_REQUIRE(id, W4_ERR_INVALID, "id buffer is required");
    W4_NCCL_API();
    static_assert(sizeof(ncclUniqueId) == W4_TP_UNIQUE_ID_BYTES, "unique id size");
    ncclUniqueId uid;
    ncclResult_t r = api.get_unique_id(&uid);
    if (r != ncclSuccess) return nccl_fail(api, r, "ncclGetUniqueId");
    memcpy(id, &uid, sizeof(uid));
    return W4_OK;
}

extern "C" int w4_tp_comm_init(w4_tp_comm **out, int nranks, int rank, const uint8_t *id, int timeout_ms) {
    set_error("");
    W4_REQUIRE(out && id, W4_ERR_INVALID, "out and id are required");
    W4_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, W4_ERR_INVALID, "rank %d of %d", rank, nranks);
    W4_REQUIRE(timeout_ms > 0, W4_ERR_INVALID, "timeout_ms must be positive");
    *out = nullptr;
    W4_NCCL_API();
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    w4_tp_comm *c = new w4_tp_comm{nullptr, nranks, rank, timeout_ms, false};
    ncclResult_t r = api.comm_init_rank_config(&c->comm, nranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return nccl_fail(api, r, "ncclCommInitRankConfig");
    }
    int rc = wait_comm_ready(api, c, timeout_ms);
    if (rc) {
        if (!c->dead) api.comm_abort(c->comm);
        delete c;
        return rc;
    }
    rc = tp_peer_setup(c);  // peer-memory all-reduce; without it NCCL carries every call
    if (rc) {
        api.comm_abort(c->comm);
        delete c;
        return rc;
    }
    *out = c;
    return W4_OK;
}

extern "C" int w4_tp_comm_destroy(w4_tp_comm *c) {
    set_error("");
    if (!c) return W4_OK;
    W4_NCCL_API();
    int rc = W4_OK;
    if (c->dead) {
        // already aborted: nothing left to release on the NCCL side
    } else {
        rc = wait_comm_ready(api, c, c->timeout_ms);  // no operation of ours still being enqueued
        if (rc) {
            delete c;
            return rc;
        }
        tp_peer_teardown(c);
        ncclResult_t r = api.comm_finalize(c->comm);
        if (r == ncclSuccess || r == ncclInProgress) rc = wait_comm_ready(api, c, c->timeout_ms);
        else rc = nccl_fail(api, r, "ncclCommFinalize");
        if (!c->dead) api.comm_destroy(c->comm);
    }
    delete c;
    return rc;
}

extern "C" int w4_tp_comm_abort(w4_tp_comm *c) {
    set_error("");
    if (!c) return W4_OK;
    W4_NCCL_API();
    if (!c->dead) api.comm_abort(c->comm);
    tp_peer_teardown(c);
    delete c;
    return W4_OK;
}

extern "C" int w4_tp_allreduce(w4_tp_comm *c, void *buf, size_t count, int dtype, void *stream) {
    set_error("");
    W4_REQUIRE(c && buf, W4_ERR_INVALID, "comm and buf are required");
    W4_REQUIRE(!c->dead, W4_ERR_INVALID, "communicator was aborted");
    W4_REQUIRE(dtype == W4_F16 || dtype == W4_BF16 || dtype == W4_F32, W4_ERR_INVALID,
               "dtype must be f16, bf16 or f32");
    W4_NCCL_API();
    if (count == 0 || c->nranks == 1) return W4_OK;
    const int rp = tp_peer_allreduce(c, buf, count, dtype, reinterpret_cast<cudaStream_t>(stream));
    if (rp >= 0) return rp;
    ncclResult_t r = api.all_reduce(buf, buf, count, nccl_dtype(dtype), ncclSum, c->comm,
                                    reinterpret_cast<cudaStream_t>(stream));
    if (r == ncclInProgress)  // a non-blocking communicator finishing the enqueue (e.g. first-use connections)
        return wait_comm_ready(api, c, c->timeout_ms);
    if (r != ncclSuccess) return nccl_fail(api, r, "ncclAllReduce");
    return W4_OK;
}

extern "C" int w4_tp_wait(w4_tp_comm *c, void *stream, int timeout_ms) {
    set_error("");
    W4_REQUIRE(c, W4_ERR_INVALID, "comm is required");
    W4_REQUIRE(!c->dead, W4_ERR_INVALID, "communicator was aborted");
    W4_REQUIRE(timeout_ms > 0, W4_ERR_INVALID, "timeout_ms must be positive");
    W4_NCCL_API();
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const auto t0 = Clock::now();
    for (;;) {
        cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) {
            // a one-shot all-reduce whose peer never pushed ended with a device status
            int rs = c->p2p ? take_tp_wait_status() : W4_OK;
            const int rf = c->p2p ? take_tp_fused_wait_status() : W4_OK;
            if (!rs) rs = rf;
            if (rs) {
                api.comm_abort(c->comm);
                c->dead = true;
            }
            return rs;
        }
        if (q != cudaErrorNotReady) {
            set_error("stream error: %s", cudaGetErrorString(q));
            return W4_ERR_CUDA;
        }
        ncclResult_t st_async = ncclSuccess;
        api.comm_get_async_error(c->comm, &st_async);
        if (st_async != ncclSuccess && st_async != ncclInProgress) {
            api.comm_abort(c->comm);
            c->dead = true;
            return nccl_fail(api, st_async, "collective");
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count() > timeout_ms) {
            api.comm_abort(c->comm);
            c->dead = true;
            set_error("stream not done after %d ms (a peer did not reach the collective); communicator aborted",
                      timeout_ms);
            return W4_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

extern "C" int w4_tp_set_fused_epilogue(w4_tp_comm *c, int on) {
    set_error("");
    W4_REQUIRE(c, W4_ERR_INVALID, "comm is required");
    c->fuse = on != 0;
    return W4_OK;
}

extern "C" size_t w4_tp_linear_workspace_bytes(int mode, int M, int N, int K, int group_size, int has_perm,
                                               int c_dtype) {
    size_t ws = w4_gptq_workspace_bytes(M, N, K, group_size, has_perm, c_dtype == W4_E4M3 ? W4_F32 : c_dtype);
    if (c_dtype == W4_E4M3) ws = (ws + 255) / 256 * 256 + (size_t)M * N * 4;  // f32 partial, reduced in place
    (void)mode;
    return ws;
}

extern "C" int w4_tp_linear(w4_tp_comm *c, int mode, const void *a, int a_dtype, const int32_t *qweight,
                            const int32_t *qzeros, const uint16_t *scales, const int32_t *perm, void *out,
                            int c_dtype, float *row_scale, int M, int N, int K, int group_size,
                            int zero_offset, void *workspace, size_t workspace_bytes, void *stream) {
    set_error("");
    W4_REQUIRE(mode == W4_TP_COLUMN || mode == W4_TP_ROW, W4_ERR_INVALID, "mode must be column or row");
    if (mode == W4_TP_COLUMN)  // this rank's N columns; no exchange
        return w4_gptq_gemm(a, a_dtype, qweight, qzeros, scales, perm, out, c_dtype, row_scale, M, N, K,
                            group_size, zero_offset, workspace, workspace_bytes, stream);
    W4_REQUIRE(c, W4_ERR_INVALID, "row-parallel needs a communicator");
    W4_REQUIRE(!c->dead, W4_ERR_INVALID, "communicator was aborted");
    const size_t need = w4_tp_linear_workspace_bytes(mode, M, N, K, group_size, perm != nullptr, c_dtype);
    W4_REQUIRE(workspace_bytes >= need && (need == 0 || workspace), W4_ERR_INVALID,
               "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    if (c->fuse && c->p2p && !perm && M <= 16) {
        // decode: the GEMM pushes its fp32 partial tiles to every rank and sums them in
        // its own epilogue (no separate all-reduce launch)
        PeerReduce pr;
        if (tp_peer_reduce_args(c, &pr)) {
            int rc = check_gptq_gemm(a, a_dtype, qweight, scales, out, c_dtype, row_scale, M, N, K, group_size);
            if (rc) return rc;
            cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
            if (c_dtype != W4_E4M3) {
                rc = gptq_gemv_tma_ar(a, a_dtype, qweight, qzeros, scales, out, c_dtype, M, N, K, group_size,
                                      zero_offset, pr, st);
                if (rc != -1) return rc;
            } else {
                const size_t gws = w4_gptq_workspace_bytes(M, N, K, group_size, 0, W4_F32);
                float *part = reinterpret_cast<float *>(static_cast<char *>(workspace) + (gws + 255) / 256 * 256);
                rc = gptq_gemv_tma_ar(a, a_dtype, qweight, qzeros, scales, part, W4_F32, M, N, K, group_size,
                                      zero_offset, pr, st);
                if (rc == W4_OK) return rowscale_fp8(part, W4_F32, static_cast<uint8_t *>(out), row_scale, M, N, st);
                if (rc != -1) return rc;
            }
        }
    }
    if (c_dtype != W4_E4M3) {
        // partial product over this rank's K rows, then the in-place sum
        int rc = w4_gptq_gemm(a, a_dtype, qweight, qzeros, scales, perm, out, c_dtype, nullptr, M, N, K,
                              group_size, zero_offset, workspace, workspace_bytes, stream);
        if (rc) return rc;
        return w4_tp_allreduce(c, out, (size_t)M * N, c_dtype, stream);
    }
    // fp8 row-scaled output: the scale needs the full sum, so reduce in f32 first
    const size_t gws = w4_gptq_workspace_bytes(M, N, K, group_size, perm != nullptr, W4_F32);
    char *wsb = static_cast<char *>(workspace);
    float *part = reinterpret_cast<float *>(wsb + (gws + 255) / 256 * 256);
    int rc = w4_gptq_gemm(a, a_dtype, qweight, qzeros, scales, perm, part, W4_F32, nullptr, M, N, K, group_size,
                          zero_offset, workspace, gws, stream);
    if (rc) return rc;
    rc = w4_tp_allreduce(c, part, (size_t)M * N, W4_F32, stream);
    if (rc) return rc;
    W4_REQUIRE(row_scale, W4_ERR_INVALID, "e4m3 output needs row_scale");
    return w4_rowscale_fp8(part, W4_F32, static_cast<uint8_t *>(out), row_scale, M, N, stream);
}
