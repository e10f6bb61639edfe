// w4_internal.h -- launchers shared between the libw4 translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "w4.h"

namespace w4 {

// gptq.cu
int gptq_dequant(const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                 const int32_t *g_idx, int K, int N, int gs, int zero_offset, float *w,
                 cudaStream_t st);
int gptq_repack_act_order(const int32_t *qweight, const int32_t *g_idx, int K, int N, int gs,
                          int32_t *qweight_out, int32_t *perm_out, cudaStream_t st);
int gather_cols(const uint16_t *a, const int32_t *perm, int M, int K, uint16_t *out,
                cudaStream_t st);
// Any M: the tensor-core GEMM for M >= kPrefillMinM when it takes the shape, else
// the decode kernels.  sync: the workspace's zeroed sync area (may be null); ws /
// ws_bytes: scratch for split-K partials (may be null: no K split).
int gptq_gemv(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
              const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs,
              int zero_offset, void *sync, void *ws, size_t ws_bytes, cudaStream_t st);
int gptq_gemv_tma(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                  const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset,
                  cudaStream_t st);
int take_wait_status();
// The workspace sync area (W4_WORKSPACE_SYNC_BYTES, zero between calls) as 32-bit words: tile
// counters from word 0, then 16 row maxima (fp32 bits of |y|) and 16 row counters at the end.
constexpr int kMaxExperts = 64;  // expert groups of one grouped (MoE) GEMM call
constexpr int kSyncWords = W4_WORKSPACE_SYNC_BYTES / 4;
constexpr int kSyncTileCounters = kSyncWords - 32;
constexpr int kSyncRowMax = kSyncWords - 32;
constexpr int kSyncRowCnt = kSyncWords - 16;
// gptq_decode.cu: the shared-ring decode GEMM (M <= 16); -1 = shape not handled there.
// sync: zeroed tile counters (W4_WORKSPACE_SYNC_BYTES); ws: K-split partials of
// gptq_decode_split_bytes() bytes.  Without them the GEMM runs unsplit.  rowmax (optional): the
// row maxima of |C| are folded into it with atomicMax on their fp32 bits.
int gptq_gemv_decode(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                     const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset,
                     void *sync, void *ws, size_t ws_bytes, unsigned int *rowmax, cudaStream_t st);
size_t gptq_decode_split_bytes(int M, int N, int K, int gs);
// gptq.cu: decode shapes that run the register-batched kernel by design (faster there)
bool prefer_register_gemv(int M, int N, int K);
// Grouped (MoE) form: expert e's weights are slice e of stacked [E][...] tensors and its token
// rows are [off[e], off[e+1]) of a and c (host offsets, off[0] = 0, at most 64 experts).
int gptq_gemv_decode_grouped(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                             const uint16_t *scales, const int *off, int n, void *c, int c_dtype, int N, int K, int gs,
                             int zero_offset, void *sync, void *ws, size_t ws_bytes, cudaStream_t st);
size_t gptq_decode_grouped_split_bytes(const int *off, int n, int N, int K, int gs);
int take_decode_wait_status();
// w4_api.cu: count a decode call that ran a register-streamed fallback kernel
void note_decode_fallback();

// Row-parallel decode GEMM with the all-reduce in its epilogue (gptq_tma.cu), over
// the peer buffers of a tensor-parallel communicator (tp_peer.cu lays them out):
// buf[p] is rank p's symmetric buffer mapped into this process.
constexpr int kPeerMaxRanks = 8;
struct PeerReduce {
    char *buf[kPeerMaxRanks];
    size_t data_off;    // fp32 partials [2 parities][nranks][slot_bytes]
    size_t slot_bytes;  // per rank and parity: M * N * 4 must fit
    size_t flags_off;   // u32 [2 parities][max_ctas][8 ranks]
    size_t ctrl_off;    // u32 {call sequence, CTAs finished}
    int rank, nranks, max_ctas;
};
// W4_OK / a W4 error, or -1 when this shape or device cannot run the fused kernel.
int gptq_gemv_tma_ar(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                     const uint16_t *scales, void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset,
                     const PeerReduce &pr, cudaStream_t st);
int take_tp_fused_wait_status();
// w4_api.cu: the argument rules of w4_gptq_gemm, without the workspace
int check_gptq_gemm(const void *a, int a_dtype, const int32_t *qweight, const uint16_t *scales, const void *c,
                    int c_dtype, const float *row_scale, int M, int N, int K, int group_size);
// gptq_prefill.cu (tcgen05); -1 = shape not handled there
int gptq_prefill(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                 void *c, int c_dtype, int M, int N, int K, int gs, int zero_offset, void *split_ws,
                 size_t split_ws_bytes, cudaStream_t st);
size_t gptq_prefill_split_bytes(int M, int N, int K, int gs, int c_dtype);
int take_prefill_wait_status();
// NVFP4 weights, bf16 activations, on the tensor cores (gptq_prefill.cu); -1 = not handled
int nvfp4_w4a16_prefill(const uint16_t *a, const uint8_t *w_nk, const uint8_t *scale, const float *w_global,
                        void *c, int c_dtype, int M, int N, int K, void *split_ws, size_t split_ws_bytes,
                        cudaStream_t st);
size_t nvfp4_w4a16_prefill_split_bytes(int M, int N, int K, int c_dtype);
// The same tensor-core GEMMs over E stacked expert matrices, rows off[e]..off[e+1] of a and c
// for expert e (gptq_prefill.cu); -1 = not handled there
int gptq_prefill_grouped(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                         const uint16_t *scales, const int *off, int n, void *c, int c_dtype, int N, int K, int gs,
                         int zero_offset, void *split_ws, size_t split_ws_bytes, cudaStream_t st);
size_t gptq_prefill_grouped_split_bytes(const int *off, int n, int N, int K, int gs, int c_dtype);
int nvfp4_w4a16_prefill_grouped(const uint16_t *a, const uint8_t *w_nk, const uint8_t *scale, const float *w_global,
                                const int *off, int n, void *c, int c_dtype, int N, int K, void *split_ws,
                                size_t split_ws_bytes, cudaStream_t st);
size_t nvfp4_w4a16_prefill_grouped_split_bytes(const int *off, int n, int N, int K, int c_dtype);
// Grouped calls whose largest expert has more rows than this run the tensor-core GEMM (each
// expert's weight tile dequantised once for up to 256 of its rows) instead of the decode kernel
// (one pass over the weights per 16 rows)
constexpr int kGroupedPrefillMinRows = 17;
constexpr int kPrefillMinM = 17;  // token counts from here on run the tensor-core prefill GEMM
// NVFP4 W4A16: the two-token-tile decode kernel (M = 9..16) is slower than the tensor-core
// GEMM, which therefore starts at 9 tokens
constexpr int kFp4PrefillMinM = 9;
// NVFP4 W4A16 calls of up to 16 tokens that run the decode kernel rather than the tensor-core
// GEMM (nvfp4_decode.cu)
bool prefer_fp4_decode(int M, int N, int K);
int gptq_s4a(const uint8_t *a, const uint8_t *b, const float *a_scale, const uint16_t *s,
             uint16_t *c, int rows, int cols, int dk, cudaStream_t st);

// nvfp4.cu
int nvfp4_dequant(const uint8_t *w, int layout, const void *scale, int scale_dtype,
                  const float *global_scale, int K, int N, float *out, cudaStream_t st);
int nvfp4_quant_act(const uint16_t *a, int M, int K, const float *a_global, uint8_t *codes,
                    uint8_t *sf, cudaStream_t st);
int nvfp4_quant_act_atoms(const uint16_t *a, int M, int K, const float *a_global, uint8_t *codes,
                          uint8_t *sf_atoms, cudaStream_t st);
int nvfp4_lut_s8a(const int8_t *a, const uint8_t *packed, const float *a_s, const float *b_s,
                  uint16_t *c, int rows, int cols, int dk, cudaStream_t st);
// nvfp4_decode.cu (shared TMA ring; K split through the workspace): -1 = not handled there
size_t nvfp4_decode_split_bytes(int M, int N, int K);
int nvfp4_gemv_decode(const uint16_t *a, const uint8_t *w, const void *scale, int scale_dtype,
                      const float *global_scale, void *c, int c_dtype, int M, int N, int K, void *sync, void *ws,
                      size_t ws_bytes, unsigned int *rowmax, cudaStream_t st);
int take_fp4d_wait_status();
int nvfp4_gemv_decode_grouped(const uint16_t *a, const uint8_t *w, const void *scale, int scale_dtype,
                              const float *global_scale, const int *off, int n, void *c, int c_dtype, int N, int K,
                              void *sync, void *ws, size_t ws_bytes, cudaStream_t st);
size_t nvfp4_decode_grouped_split_bytes(const int *off, int n, int N, int K);
// nvfp4_prefill.cu (tcgen05 block-scaled); -1 = shape not handled there
size_t nvfp4_prefill_workspace(int M, int N, int K);
int nvfp4_prefill(const uint16_t *a, const float *a_global, const uint8_t *w_nk, const uint8_t *w_sf,
                  bool w_sf_atoms, const float *w_global, void *c, int c_dtype, int M, int N, int K,
                  void *workspace, cudaStream_t st);
int nvfp4_sf_atoms(const uint8_t *src, int rows, int nkb, long rs, long ks, uint8_t *dst, cudaStream_t st);
int take_fp4_prefill_wait_status();
// sync / ws / ws_bytes: the workspace's sync area and the space for K-split partials (null:
// no K split)
int nvfp4_gemv(const uint16_t *a, const uint8_t *w, int layout, const void *scale,
               int scale_dtype, const float *global_scale, void *c, int c_dtype, int M, int N,
               int K, void *sync, void *ws, size_t ws_bytes, cudaStream_t st);

// epilogue.cu
int rmsnorm_quant_s8(const uint16_t *x, int8_t *q, float *scale, int M, int K, float eps,
                     cudaStream_t st);
int take_rn_wait_status();
// RMSNorm -> NVFP4 codes [rows, K/2] + scale atoms, rows = M rounded up to 128 (nvfp4.cu).
int rmsnorm_nvfp4(const void *x, int x_dtype, const void *gamma, float eps, const float *a_global, uint8_t *codes,
                  uint8_t *sf_atoms, int M, int K, cudaStream_t st);
// The block-scaled GEMM from quantised activations (nvfp4_prefill.cu).
int nvfp4_prefill_q(const uint8_t *codes, const uint8_t *sfa, const float *a_global, const uint8_t *w_nk,
                    const uint8_t *w_sf, bool w_sf_atoms, const float *w_global, void *c, int c_dtype, int M, int N,
                    int K, void *workspace, cudaStream_t st);
size_t nvfp4_prefill_q_workspace(int M, int N, int K, bool scale_atoms_needed);
// C = sum over splits of the fp32 partials [splits][mn] (mn % 4 == 0), in c_dtype (gptq_prefill.cu).
int splitk_reduce(const float *partial, int splits, long mn, void *c, int c_dtype, cudaStream_t st);
int rowscale_fp8(const void *y, int y_dtype, uint8_t *q, float *row_scale, int M, int N,
                 cudaStream_t st);
// The same cast (bit for bit) from f32 y whose row maxima a decode GEMM folded into rowmax (fp32
// bits, M <= 16); the last CTA of each row zeroes rowmax[row] again, counting on rowcnt[row].
int rowscale_fp8_amax(const float *y, unsigned int *rowmax, unsigned int *rowcnt, uint8_t *q, float *row_scale,
                      int M, int N, cudaStream_t st);

}  // namespace w4
