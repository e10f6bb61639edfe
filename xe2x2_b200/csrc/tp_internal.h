// tp_internal.h -- the tensor-parallel communicator shared by tp.cu (NCCL side)
// and tp_peer.cu (one-shot all-reduce over peer memory).
#pragma once
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdint.h>

#include <mutex>

#include "w4_internal.h"

constexpr int kTpMaxRanks = 8;

struct w4_tp_comm {
    ncclComm_t comm;
    int nranks, rank;
    int timeout_ms;  // bound on every host-side wait for this communicator
    bool dead;
    // One-shot all-reduce over peer memory (tp_peer.cu).  sym is this rank's
    // symmetric buffer (slots, flags, block counters); peer[p] is rank p's
    // buffer mapped into this process (peer[rank] == sym).  p2p is false when
    // the buffers could not be mapped; NCCL then carries every all-reduce.
    void *sym = nullptr;
    void *peer[kTpMaxRanks] = {};
    bool p2p = false;
    bool fuse = false;  // row-parallel decode GEMMs reduce in their own epilogue (w4_tp_set_fused_epilogue)
};

namespace w4 {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*comm_abort)(ncclComm_t);
    ncclResult_t (*comm_finalize)(ncclComm_t);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    const char *(*error_string)(ncclResult_t);
    bool ok;
};

// NCCL resolved at run time: the copy the process already loaded, else the
// system libnccl.so.2.
inline const NcclApi &nccl() {
    static NcclApi api{};
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto sym = [&](const char *n) { return dlsym(h, n); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank_config =
            reinterpret_cast<decltype(api.comm_init_rank_config)>(sym("ncclCommInitRankConfig"));
        api.comm_get_async_error =
            reinterpret_cast<decltype(api.comm_get_async_error)>(sym("ncclCommGetAsyncError"));
        api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
        api.comm_finalize = reinterpret_cast<decltype(api.comm_finalize)>(sym("ncclCommFinalize"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank_config && api.comm_get_async_error &&
                 api.comm_abort && api.comm_finalize && api.comm_destroy && api.all_reduce &&
                 api.all_gather && api.error_string;
    });
    return api;
}

// tp_peer.cu
int tp_peer_setup(w4_tp_comm *c);                  // after the NCCL communicator is ready
void tp_peer_teardown(w4_tp_comm *c);              // unmap peers, free the local buffer
// W4_OK / a W4 error, or -1 when the one-shot path does not take this call.
int tp_peer_allreduce(w4_tp_comm *c, void *buf, size_t count, int dtype, cudaStream_t st);
int take_tp_wait_status();
// The peer buffers as the fused row-parallel GEMM sees them; false without the peer path.
bool tp_peer_reduce_args(const w4_tp_comm *c, PeerReduce *pr);

}  // namespace w4
