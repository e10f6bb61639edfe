// tp_peer.cu -- one-shot all-reduce of row-parallel partial outputs over peer
// memory (NVLink / NVSwitch), for the small messages of decode-sized layers.
//
// Every rank owns a symmetric buffer, exported with CUDA IPC and mapped into
// every other rank at communicator creation (the handles travel by an NCCL
// all-gather).  Layout (kTpSlotBytes per slot):
//   data   [2 parities][nranks][kTpSlotBytes]   partials pushed by each rank
//   flags  [2 parities][kTpMaxBlocks][8] u32   "block b of rank p has pushed"
//   ctr    [kTpMaxBlocks] u32                   this rank's per-block call counter
// A call runs one CTA per chunk of the message.  CTA b reads its counter
// (v = ctr[b] + 1, parity v & 1), stores its chunk of the local partial into
// slot[parity][rank] of every rank's buffer, fences at system scope, raises
// flag[parity][b][rank] = v on every rank (st.release.sys), waits until its
// own flags [parity][b][p] == v for every p (ld.acquire.sys, bounded by a time
// limit), then sums slot[parity][0 .. nranks-1] in rank order into the output
// (identical bits on every rank) and stores ctr[b] = v.
// Reuse is safe with two parities: a rank can only be one call ahead of a peer
// still reading, because each call waits for every peer's push of that call.
// The counters live in device memory, so captured CUDA graphs replay correctly.
// No copy here is a TMA or bulk load, and nothing uses multicast.
// Messages up to 512 KB (decode-sized outputs) take a second form that needs
// neither the fence nor the flags: every 4-byte word travels with the call
// number in one 8-byte store and readers wait on the words themselves (see
// ll_off).  The same buffer also carries the epilogue all-reduce of the fused
// row-parallel decode GEMM (separate slots, flags and sequence; see fdata_off).
#include <chrono>
#include <thread>

#include "tp_internal.h"
#include "w4_common.cuh"
#include "w4_internal.h"

namespace w4 {

static __device__ unsigned int g_tp_timeout;  // a peer never pushed within the time limit (sticky)

constexpr size_t kTpSlotBytes = size_t(1) << 20;  // largest one-shot message per rank
constexpr int kTpMaxBlocks = 64;
constexpr int kTpThreads = 256;
constexpr unsigned long long kTpWaitNs = 500ull * 1000 * 1000;  // 500 ms

static size_t flags_off(int nranks) { return 2 * (size_t)nranks * kTpSlotBytes; }
static size_t ctr_off(int nranks) { return flags_off(nranks) + 2 * kTpMaxBlocks * 8 * sizeof(uint32_t); }

// A second region serves the row-parallel decode GEMM that reduces in its own
// epilogue (gptq_tma.cu): its own fp32 slots, per-CTA flags and a control word
// pair {call sequence, CTAs finished}, so its parity sequence never shares
// slots with the all-reduce kernel's.
constexpr size_t kFusedSlotBytes = size_t(512) << 10;  // M * N * 4 per rank and parity
constexpr int kFusedMaxCtas = 1024;
static size_t fdata_off(int nranks) { return (ctr_off(nranks) + kTpMaxBlocks * sizeof(uint32_t) + 255) & ~size_t(255); }
static size_t fflags_off(int nranks) { return fdata_off(nranks) + 2 * (size_t)nranks * kFusedSlotBytes; }
static size_t fctrl_off(int nranks) { return fflags_off(nranks) + 2 * (size_t)kFusedMaxCtas * 8 * sizeof(uint32_t); }

// A third region carries small messages (up to kLLMaxBytes) with the data and the call number
// side by side: every 4-byte word of a partial travels as one 8-byte store {word, v}, and a
// reader takes a word once its v matches, so no fence or separate flag is needed (an aligned
// 8-byte store is observed whole).  Layout: slots [2 parities][nranks][kLLSlotBytes], then
// this rank's call sequence and finished-block count.
constexpr size_t kLLMaxBytes = size_t(512) << 10;
constexpr size_t kLLSlotBytes = 2 * kLLMaxBytes;  // 8 bytes per 4-byte word
constexpr int kLLWordsPerBlock = 2048;
static size_t ll_off(int nranks) { return (fctrl_off(nranks) + 256 + 255) & ~size_t(255); }
static size_t llctr_off(int nranks) { return ll_off(nranks) + 2 * (size_t)nranks * kLLSlotBytes; }
static size_t sym_bytes(int nranks) { return llctr_off(nranks) + kTpMaxBlocks * sizeof(uint32_t) + 256; }

struct PeerPtrs {
    char *p[kTpMaxRanks];
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long tp_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

template <typename T> struct Acc;
template <> struct Acc<__nv_bfloat16> {
    static __device__ float to(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __nv_bfloat16 from(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Acc<__half> {
    static __device__ float to(__half x) { return __half2float(x); }
    static __device__ __half from(float x) { return __float2half_rn(x); }
};
template <> struct Acc<float> {
    static __device__ float to(float x) { return x; }
    static __device__ float from(float x) { return x; }
};

// n is a multiple of 16 / sizeof(T); every block owns whole 16-byte vectors.
template <typename T>
__global__ void __launch_bounds__(kTpThreads)
oneshot_allreduce_kernel(PeerPtrs pp, int rank, int nranks, T *__restrict__ data, long n, long per_block,
                         size_t foff, size_t coff) {
    constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
    const int b = blockIdx.x;
    const long i0 = b * per_block, i1 = min(n, i0 + per_block);
    uint32_t *ctr = reinterpret_cast<uint32_t *>(pp.p[rank] + coff) + b;
    __shared__ uint32_t v_s;
    if (threadIdx.x == 0) v_s = *ctr + 1;
    __syncthreads();
    const uint32_t v = v_s;
    const int par = v & 1;

    // 1. push this rank's chunk into slot [par][rank] of every rank
    for (long i = i0 + threadIdx.x * V; i < i1; i += kTpThreads * V) {
        const uint4 x = *reinterpret_cast<const uint4 *>(data + i);
        for (int p = 0; p < nranks; ++p) {
            T *slot = reinterpret_cast<T *>(pp.p[p] + (size_t)(par * nranks + rank) * kTpSlotBytes);
            *reinterpret_cast<uint4 *>(slot + i) = x;
        }
    }
    __syncthreads();
    // the system fence and release of the flagging threads are cumulative over the barrier
    if (threadIdx.x < nranks) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t *>(pp.p[threadIdx.x] + foff) + (par * kTpMaxBlocks + b) * 8 + rank, v);
    }

    // 2. wait until every rank has pushed block b of this call into this rank's buffer
    if (threadIdx.x < nranks) {
        const uint32_t *f = reinterpret_cast<const uint32_t *>(pp.p[rank] + foff) + (par * kTpMaxBlocks + b) * 8 +
                            threadIdx.x;
        if (ld_acquire_sys(f) != v) {
            const unsigned long long t0 = tp_ns();
            while (ld_acquire_sys(f) != v) {
                if (tp_ns() - t0 > kTpWaitNs) {
                    atomicExch(&g_tp_timeout, 1u);
                    break;
                }
            }
        }
    }
    __syncthreads();

    // 3. sum the nranks slots in rank order (same bits on every rank), through L2
    for (long i = i0 + threadIdx.x * V; i < i1; i += kTpThreads * V) {
        float acc[V];
#pragma unroll
        for (int e = 0; e < V; ++e) acc[e] = 0.f;
        for (int p = 0; p < nranks; ++p) {
            const T *slot = reinterpret_cast<const T *>(pp.p[rank] + (size_t)(par * nranks + p) * kTpSlotBytes);
            const uint4 x = __ldcg(reinterpret_cast<const uint4 *>(slot + i));
            const T *e8 = reinterpret_cast<const T *>(&x);
#pragma unroll
            for (int e = 0; e < V; ++e) acc[e] += Acc<T>::to(e8[e]);
        }
        uint4 y;
        T *o = reinterpret_cast<T *>(&y);
#pragma unroll
        for (int e = 0; e < V; ++e) o[e] = Acc<T>::from(acc[e]);
        *reinterpret_cast<uint4 *>(data + i) = y;
    }
    __syncthreads();
    if (threadIdx.x == 0) *ctr = v;
}

// ---- the small-message form: data and call number in one 8-byte store ----
__device__ __forceinline__ void st_ll(char *p, uint32_t d, uint32_t f) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(d), "r"(f) : "memory");
}
__device__ __forceinline__ uint2 ld_ll(const char *p) {
    uint2 r;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
    return r;
}

// A 4-byte word of T values, summed in fp32 and rounded back as the one-shot kernel does.
template <typename T> struct Word {
    static constexpr int E = 4 / sizeof(T);
    static __device__ void add(float (&acc)[E], uint32_t w) {
        const T *e = reinterpret_cast<const T *>(&w);
#pragma unroll
        for (int i = 0; i < E; ++i) acc[i] += Acc<T>::to(e[i]);
    }
    static __device__ uint32_t pack(const float (&acc)[E]) {
        uint32_t w;
        T *e = reinterpret_cast<T *>(&w);
#pragma unroll
        for (int i = 0; i < E; ++i) e[i] = Acc<T>::from(acc[i]);
        return w;
    }
};

// One call number per call, the same in every block: v = seq + 1 (parity v & 1), where seq
// (ctl[0]) advances once the last block of the call is done (ctl[1] counts finished blocks), so
// a word of an older call always carries an older number, whichever block moved it (the
// word-to-block partition changes with the message size).  Block b owns words
// [b * per_block, ...): each thread stores {word, v} of its words into slot [parity][rank] of
// every rank, then sums slot [parity][0 .. nranks-1] of the same words in rank order as each
// reads v (bounded by the time limit; after one expiry a thread stops waiting).  A thread
// reads back only the words it wrote itself in its own slot.  Reuse of a parity is safe as in
// the one-shot kernel: a rank is at most one call ahead of a peer still reading.
template <typename T>
__global__ void __launch_bounds__(kTpThreads)
ll_allreduce_kernel(PeerPtrs pp, int rank, int nranks, T *__restrict__ data, long nwords, long per_block,
                    size_t loff, size_t coff) {
    const int b = blockIdx.x;
    const long w0 = b * per_block, w1 = min(nwords, w0 + per_block);
    uint32_t *ctl = reinterpret_cast<uint32_t *>(pp.p[rank] + coff);  // {call sequence, blocks done}
    __shared__ uint32_t v_s;
    if (threadIdx.x == 0) v_s = *reinterpret_cast<volatile uint32_t *>(ctl) + 1;
    __syncthreads();
    const uint32_t v = v_s;
    const int par = v & 1;
    uint32_t *words = reinterpret_cast<uint32_t *>(data);
    for (long w = w0 + threadIdx.x; w < w1; w += kTpThreads) {
        const uint32_t x = words[w];
        for (int p = 0; p < nranks; ++p)
            st_ll(pp.p[p] + loff + (size_t)(par * nranks + rank) * kLLSlotBytes + (size_t)w * 8, x, v);
    }
    bool waiting = true;
    for (long w = w0 + threadIdx.x; w < w1; w += kTpThreads) {
        float acc[Word<T>::E];
#pragma unroll
        for (int i = 0; i < Word<T>::E; ++i) acc[i] = 0.f;
        for (int p = 0; p < nranks; ++p) {
            const char *slot = pp.p[rank] + loff + (size_t)(par * nranks + p) * kLLSlotBytes + (size_t)w * 8;
            uint2 r = ld_ll(slot);
            if (r.y != v && waiting) {
                const unsigned long long t0 = tp_ns();
                while ((r = ld_ll(slot)).y != v) {
                    if (tp_ns() - t0 > kTpWaitNs) {
                        atomicExch(&g_tp_timeout, 1u);
                        waiting = false;
                        break;
                    }
                }
            }
            Word<T>::add(acc, r.x);
        }
        words[w] = Word<T>::pack(acc);
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(&ctl[1], 1u) == gridDim.x - 1) {  // every block has read seq
        ctl[1] = 0;
        ctl[0] = v;
    }
}

static int wait_stream_bounded(cudaStream_t st, int timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) return W4_OK;
        if (q != cudaErrorNotReady) {
            set_error("stream error: %s", cudaGetErrorString(q));
            return W4_ERR_CUDA;
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() >
            timeout_ms) {
            set_error("peer buffer exchange not done after %d ms", timeout_ms);
            return W4_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

// A non-blocking communicator may still be finishing the enqueue of the last
// call (ncclInProgress); NCCL accepts the next call only once that is done.
static int settle(const NcclApi &api, w4_tp_comm *c) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = api.comm_get_async_error(c->comm, &st);
        if (r != ncclSuccess || (st != ncclSuccess && st != ncclInProgress)) {
            set_error("NCCL communicator error %d / %d", (int)r, (int)st);
            return W4_ERR_NCCL;
        }
        if (st == ncclSuccess) return W4_OK;
        if (std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() >
            c->timeout_ms) {
            set_error("NCCL call not enqueued after %d ms", c->timeout_ms);
            return W4_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

// Export this rank's buffer, all-gather the handles over NCCL, map the peers'.
// Any failure to map leaves p2p off (NCCL carries the all-reduces); only an
// NCCL error or timeout during the exchange is reported.
int tp_peer_setup(w4_tp_comm *c) {
    c->p2p = false;
    if (c->nranks < 2 || c->nranks > kTpMaxRanks) return W4_OK;
    const NcclApi &api = nccl();
    const size_t bytes = sym_bytes(c->nranks);
    if (cudaMalloc(&c->sym, bytes) != cudaSuccess) {
        cudaGetLastError();
        c->sym = nullptr;
        return W4_OK;
    }
    W4_CUDA_TRY(cudaMemset(c->sym, 0, bytes));
    cudaIpcMemHandle_t mine;
    memset(&mine, 0, sizeof(mine));
    const bool exported = cudaIpcGetMemHandle(&mine, c->sym) == cudaSuccess;
    if (!exported) cudaGetLastError();
    // every rank takes part in the exchange (a zero handle marks "no export")
    constexpr size_t H = sizeof(cudaIpcMemHandle_t);
    uint8_t *dev = nullptr;
    W4_CUDA_TRY(cudaMalloc(&dev, H * (c->nranks + 1)));
    cudaStream_t st;
    W4_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    W4_CUDA_TRY(cudaMemcpy(dev + H * c->nranks, &mine, H, cudaMemcpyHostToDevice));
    ncclResult_t r = api.all_gather(dev + H * c->nranks, dev, H, ncclUint8, c->comm, st);
    int rc = W4_OK;
    if (r != ncclSuccess && r != ncclInProgress) {
        set_error("ncclAllGather of peer handles: %s", api.error_string(r));
        rc = W4_ERR_NCCL;
    } else {
        rc = settle(api, c);
        if (!rc) rc = wait_stream_bounded(st, c->timeout_ms);
    }
    uint8_t all[H * kTpMaxRanks];
    if (!rc) rc = cudaMemcpy(all, dev, H * c->nranks, cudaMemcpyDeviceToHost) == cudaSuccess ? W4_OK : W4_ERR_CUDA;
    cudaStreamDestroy(st);
    cudaFree(dev);
    if (rc) return rc;
    bool ok = exported;
    for (int p = 0; p < c->nranks; ++p) {
        if (p == c->rank) {
            c->peer[p] = c->sym;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, all + H * p, H);
        static const cudaIpcMemHandle_t zero{};
        if (!memcmp(&h, &zero, H) || cudaIpcOpenMemHandle(&c->peer[p], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            c->peer[p] = nullptr;
            ok = false;
        }
    }
    // Every rank must agree on using the peer path: all-reduce the decisions.
    int *flag = nullptr;
    W4_CUDA_TRY(cudaMalloc(&flag, sizeof(int)));
    const int mine_ok = ok ? 1 : 0;
    W4_CUDA_TRY(cudaMemcpy(flag, &mine_ok, sizeof(int), cudaMemcpyHostToDevice));
    W4_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    r = api.all_reduce(flag, flag, 1, ncclInt32, ncclMin, c->comm, st);
    if (r != ncclSuccess && r != ncclInProgress) {
        set_error("ncclAllReduce of the peer-path decisions: %s", api.error_string(r));
        rc = W4_ERR_NCCL;
    } else {
        rc = settle(api, c);
        if (!rc) rc = wait_stream_bounded(st, c->timeout_ms);
    }
    int all_ok = 0;
    if (!rc) rc = cudaMemcpy(&all_ok, flag, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess ? W4_OK : W4_ERR_CUDA;
    cudaStreamDestroy(st);
    cudaFree(flag);
    if (rc) return rc;
    c->p2p = all_ok == 1;
    return W4_OK;
}

void tp_peer_teardown(w4_tp_comm *c) {
    for (int p = 0; p < kTpMaxRanks; ++p) {
        if (c->peer[p] && p != c->rank) cudaIpcCloseMemHandle(c->peer[p]);
        c->peer[p] = nullptr;
    }
    if (c->sym) cudaFree(c->sym);
    c->sym = nullptr;
    c->p2p = false;
    cudaGetLastError();
}

int tp_peer_allreduce(w4_tp_comm *c, void *buf, size_t count, int dtype, cudaStream_t st) {
    if (!c->p2p) return -1;
    const size_t es = dtype == W4_F32 ? 4 : 2;
    if (count * es > kTpSlotBytes || (count * es) % 16 || (reinterpret_cast<uintptr_t>(buf) & 15)) return -1;
    PeerPtrs pp;
    for (int p = 0; p < kTpMaxRanks; ++p) pp.p[p] = static_cast<char *>(c->peer[p]);
    if (count * es <= kLLMaxBytes) {  // data and call number side by side: no fence, no flags
        const long nwords = (long)(count * es / 4);
        const long lblocks = (nwords + kLLWordsPerBlock - 1) / kLLWordsPerBlock;
        const long lper = (nwords + lblocks - 1) / lblocks;
        const size_t lo = ll_off(c->nranks), lc = llctr_off(c->nranks);
        if (dtype == W4_BF16)
            ll_allreduce_kernel<__nv_bfloat16><<<(unsigned)lblocks, kTpThreads, 0, st>>>(
                pp, c->rank, c->nranks, static_cast<__nv_bfloat16 *>(buf), nwords, lper, lo, lc);
        else if (dtype == W4_F16)
            ll_allreduce_kernel<__half><<<(unsigned)lblocks, kTpThreads, 0, st>>>(
                pp, c->rank, c->nranks, static_cast<__half *>(buf), nwords, lper, lo, lc);
        else
            ll_allreduce_kernel<float><<<(unsigned)lblocks, kTpThreads, 0, st>>>(
                pp, c->rank, c->nranks, static_cast<float *>(buf), nwords, lper, lo, lc);
        W4_LAUNCH_CHECK();
        return W4_OK;
    }
    const long n = (long)count;
    const long v = 16 / (long)es;
    long blocks = (n + 4095) / 4096;
    if (blocks < 1) blocks = 1;
    if (blocks > kTpMaxBlocks) blocks = kTpMaxBlocks;
    long per = (n + blocks - 1) / blocks;
    per = (per + v - 1) / v * v;  // whole 16-byte vectors per block
    blocks = (n + per - 1) / per;
    const size_t fo = flags_off(c->nranks), co = ctr_off(c->nranks);
    if (dtype == W4_BF16)
        oneshot_allreduce_kernel<__nv_bfloat16><<<(unsigned)blocks, kTpThreads, 0, st>>>(
            pp, c->rank, c->nranks, static_cast<__nv_bfloat16 *>(buf), n, per, fo, co);
    else if (dtype == W4_F16)
        oneshot_allreduce_kernel<__half><<<(unsigned)blocks, kTpThreads, 0, st>>>(
            pp, c->rank, c->nranks, static_cast<__half *>(buf), n, per, fo, co);
    else
        oneshot_allreduce_kernel<float><<<(unsigned)blocks, kTpThreads, 0, st>>>(
            pp, c->rank, c->nranks, static_cast<float *>(buf), n, per, fo, co);
    W4_LAUNCH_CHECK();
    return W4_OK;
}

bool tp_peer_reduce_args(const w4_tp_comm *c, PeerReduce *pr) {
    if (!c->p2p || c->nranks > kPeerMaxRanks) return false;
    for (int p = 0; p < kPeerMaxRanks; ++p) pr->buf[p] = static_cast<char *>(c->peer[p]);
    pr->data_off = fdata_off(c->nranks);
    pr->slot_bytes = kFusedSlotBytes;
    pr->flags_off = fflags_off(c->nranks);
    pr->ctrl_off = fctrl_off(c->nranks);
    pr->rank = c->rank;
    pr->nranks = c->nranks;
    pr->max_ctas = kFusedMaxCtas;
    return true;
}

int take_tp_wait_status() {
    unsigned int v = 0;
    W4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_tp_timeout, sizeof(v)));
    if (v) {
        const unsigned int zero = 0;
        W4_CUDA_TRY(cudaMemcpyToSymbol(g_tp_timeout, &zero, sizeof(zero)));
        set_error("a peer never pushed its part of a one-shot all-reduce within the time limit");
        return W4_ERR_TIMEOUT;
    }
    return W4_OK;
}

}  // namespace w4
