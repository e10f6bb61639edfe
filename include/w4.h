/*
 * w4.h -- C ABI of libw4, the B200 (sm_100a) weight-only quantized linear
 * library (GPTQ int4 W4A16, NVFP4, epilogue quant).
 *
 * Conventions for every entry point:
 *   - All tensor pointers are DEVICE pointers unless the comment says otherwise.
 *     Row-major, densely packed, shapes as documented.  fp16 / bf16 values are
 *     passed as uint16_t bit patterns.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Work is
 *     enqueued asynchronously; the call returns once it is launched.
 *   - Nothing is allocated inside a call.  Scratch space, where needed, is the
 *     caller's `workspace` buffer, sized by the matching *_workspace_bytes().
 *     Every workspace begins with a sync area of W4_WORKSPACE_SYNC_BYTES bytes
 *     (counters of the decode GEMMs' K split).  It must be all zero before the
 *     workspace is first used; every call that completes leaves it zero, so a
 *     workspace zeroed once stays usable for any later call.  After a call
 *     whose kernel reported W4_ERR_TIMEOUT (w4_check_device_status), zero it
 *     again.
 *   - Argument errors are reported synchronously (W4_ERR_INVALID /
 *     W4_ERR_UNSUPPORTED) before anything is launched; launch failures are
 *     W4_ERR_CUDA.  w4_last_error() gives a one-line reason (thread-local).
 *   - Calls are reentrant; concurrent calls on different streams must not
 *     share a workspace.
 *
 * Each entry point names the reference (hotschmoe/xe2x2) interface it replaces,
 * as file:line within that project.  The reference's kernels are file-local
 * `sycl::event launch(sycl::queue&, ...)` functions driven by their own
 * run_shape(); its only operator-level API is the external PyTorch op
 * `torch.ops._xpu_C.nvfp4_gemm_w4a16[_f8scale]` (kernels/nvfp4/bench_nvfp4_m1.py:67,88).
 */
#ifndef W4_H
#define W4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Size of the zero-initialised sync area at the start of every workspace. */
#define W4_WORKSPACE_SYNC_BYTES 16384

#define W4_ABI_VERSION 1

/* Status codes.  The reference harness exits 0 ok / 1 numeric fail / 2 bad
 * shape or usage (kernels/esimd_dpas/dpas_s4_gptq.cpp:171-176,282-289); here a
 * bad shape is W4_ERR_INVALID and a legal-but-unsupported one W4_ERR_UNSUPPORTED. */
enum w4_status {
    W4_OK = 0,
    W4_ERR_INVALID = 1,
    W4_ERR_UNSUPPORTED = 2,
    W4_ERR_CUDA = 3,
    W4_ERR_TIMEOUT = 4,
    W4_ERR_NCCL = 5
};

/* Element types. */
enum w4_dtype {
    W4_F16 = 0,
    W4_BF16 = 1,
    W4_F32 = 2,
    W4_E4M3 = 3, /* fp8 e4m3fn (bias 7, max 448, no inf) */
    W4_S8 = 4,
    W4_E4M3_ATOMS = 5 /* NVFP4 block scales already rearranged by w4_nvfp4_repack_scales */
};

/* NVFP4 packed-weight layouts (two E2M1 nibbles per byte, low nibble = even k). */
enum w4_nvfp4_layout {
    W4_NVFP4_KN = 0, /* u8 [K/2, N], N contiguous: kernels/nvfp4/nibble_lut_sc.cpp:77-83 */
    W4_NVFP4_NK = 1  /* u8 [N, K/2], K contiguous: the external op's w with stride(0)==1,
                        kernels/nvfp4/bench_nvfp4_m1.py:58-61 */
};

/* NVFP4 activation handling. */
enum w4_act_mode {
    W4_ACT_W4A16 = 0, /* activations stay bf16; weights dequantised on the fly */
    W4_ACT_NVFP4 = 1  /* activations quantised to NVFP4 per 16-block (w4_nvfp4_quant_act) */
};

int w4_abi_version(void);
const char *w4_status_string(int status);
const char *w4_last_error(void);

/* Kernels that wait on asynchronous copies (mbarrier waits) bound every wait;
 * if one expires the kernel stops that part of its work and sets a device
 * status word.  This call reads and clears it for the current device:
 * W4_ERR_TIMEOUT if a wait expired since the last call, else W4_OK.  It
 * synchronises with the device.  No counterpart in the reference (its kernels
 * have no device-side waits). */
int w4_check_device_status(void);

/* How the decode GEMMs (the TMA-streamed M <= 16 kernels) are ordered behind
 * the previous kernel on the stream (programmatic dependent launch).
 * Process-wide; no counterpart in the reference, whose operators launch plainly.
 *   W4_OVERLAP_OFF             plain launches.
 *   W4_OVERLAP_DEPENDENT       (default) the GEMM may be scheduled while the
 *                              previous kernel drains; it sets up its barriers
 *                              and reads nothing until that kernel completed.
 *   W4_OVERLAP_STATIC_WEIGHTS  as above, and it also starts streaming the
 *                              weight operands (qweight, scales, zeros / NVFP4
 *                              codes and block scales) before then, on calls
 *                              where that measured faster (at most 16 MB of
 *                              codes and four token rows per block).  Only for
 *                              callers whose weights are never written by the
 *                              kernel that precedes the GEMM on the stream
 *                              (inference on loaded checkpoints). */
enum w4_overlap {
    W4_OVERLAP_OFF = 0,
    W4_OVERLAP_DEPENDENT = 1,
    W4_OVERLAP_STATIC_WEIGHTS = 2
};
int w4_set_launch_overlap(int mode);
int w4_get_launch_overlap(void);

/* Number of decode GEMM calls (GPTQ or NVFP4 W4A16, M <= 16) made by this process that
 * ran a register-streamed fallback kernel because none of the TMA-streamed decode kernels
 * takes the shape (for example a column count that is not a multiple of 32 for the NVFP4
 * decode kernel).  Those run correctly but 2-3x slower; benchmarks and tests assert the
 * count stays 0 on the shapes they measure.  No counterpart in the reference. */
unsigned long long w4_decode_fallback_count(void);

/* Measurement helper; no counterpart in the reference.  One launch that reads
 * `bytes` (a positive multiple of 16) of device memory at `buf` (16-byte
 * aligned) with 16-byte loads at full occupancy and writes `sink` (4 bytes of
 * device memory) only if the XOR of every word equals a fixed sentinel.  Timed
 * back to back over buffers larger than L2, it gives the read bandwidth that a
 * single kernel of that size attains on this GPU, launch ramp and tail
 * included: the practical ceiling of a decode GEMM that reads its operands
 * once.  Argument errors are synchronous (W4_ERR_INVALID). */
int w4_read_probe(const void *buf, size_t bytes, unsigned int *sink, void *stream);

/* ===================================================================== */
/* GPTQ int4                                                              */
/* ===================================================================== */

/* Dequantise a GPTQ checkpoint matrix to fp32, bit-exact:
 *   w[k,n] = float(scales[g,n]) * (q[k,n] - zero[g,n]),  g = g_idx ? g_idx[k] : k/group_size
 * qweight i32 [K/8,N] (8 nibbles LSB-first along K), qzeros i32 [K/gs,N/8]
 * (LSB-first along N) or NULL (symmetric, zero = 8), scales f16 [K/gs,N],
 * g_idx i32 [K] or NULL.  zero = stored + zero_offset (1 = GPTQ v1 "+1", 0 = v2).
 * Replaces the host unpack of kernels/nvfp4/gptq_s4_dump.py:61-73,106-114. */
int w4_gptq_dequant(const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                    const int32_t *g_idx, int K, int N, int group_size, int zero_offset,
                    float *w, void *stream);

/* act_order load-time repack: perm = stable argsort(g_idx) (i32 [K]) and
 * qweight_out[K/8,N] whose row j is row perm[j] of qweight, so every group is a
 * contiguous run of group_size rows.  Requires every group to hold exactly
 * group_size rows (GPTQ act_order does).  qweight_out must not alias qweight.
 * Replaces the g_idx check of kernels/nvfp4/gptq_s4_dump.py:119-122. */
int w4_gptq_repack_act_order(const int32_t *qweight, const int32_t *g_idx, int K, int N,
                             int group_size, int32_t *qweight_out, int32_t *perm_out,
                             void *stream);

/* Workspace needed by w4_gptq_gemm for these arguments: the sync area, plus the
 * gathered activations (act_order), the f32 product (W4_E4M3 output) and the
 * K-split partials.  At decode sizes (M <= 16) a workspace smaller than this
 * still works if it holds the sync area: the GEMM then runs without a K split
 * (correct, slower on narrow layers). */
size_t w4_gptq_workspace_bytes(int M, int N, int K, int group_size, int has_perm, int c_dtype);

/* W4A16 GPTQ GEMM:  C[m,n] = sum_k A[m,k'] * w[k,n]   (fp32 accumulate)
 * a: [M,K] f16 or bf16 (a_dtype); qweight/qzeros/scales as in w4_gptq_dequant
 * with groups contiguous (k/group_size); perm: i32 [K] from
 * w4_gptq_repack_act_order (then k' = perm[k]) or NULL (k' = k).
 * c: [M,N] of c_dtype W4_F16 / W4_BF16 / W4_F32, or W4_E4M3 with the per-row
 * scale written to row_scale f32 [M] (c = e4m3(y / row_scale), row_scale =
 * max|y_row| / 448, the epilogue_quant contract of
 * kernels/epilogue_quant/rmsnorm_epilogue.cpp:56-69 with qmax 448).
 * Shapes: K % 32 == 0, N % 32 == 0, group_size % 32 == 0, K % group_size == 0, M >= 1.
 * Replaces launch() of kernels/esimd_dpas/dpas_s4_gptq_sc.cpp:146-233 (decode)
 * and kernels/esimd_dpas/dpas_s4_gptq_db48.cpp:148-246 (prefill). */
int w4_gptq_gemm(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                 const uint16_t *scales, const int32_t *perm, void *c, int c_dtype,
                 float *row_scale, int M, int N, int K, int group_size, int zero_offset,
                 void *workspace, size_t workspace_bytes, void *stream);

/* w4_gptq_gemm with c_dtype == W4_E4M3 for callers that cannot allocate
 * device memory (a binding that only forwards pointers it was given, a runtime
 * that pre-reserved all HBM).  It has no counterpart in the reference.  Same
 * arguments and results as w4_gptq_gemm(a, a_dtype, qweight, qzeros, scales,
 * NULL, q_out, W4_E4M3, row_scale, M, N, K, group_size, zero_offset, ...), but
 * the f32 intermediate lives in a static device array inside the library
 * (4 MiB per device, held until exit) instead of a workspace: M*N must be
 * <= 1,048,576 or the call returns W4_ERR_UNSUPPORTED.  The first call on a
 * device looks the array's address up; make it before any stream capture.  The
 * address is cached per device for the life of the process: after
 * cudaDeviceReset on a device, do not call this on that device again.
 * All calls share the array: calls that overlap on the GPU race.  With no
 * workspace the GEMM never splits K, so results equal w4_gptq_gemm's only to
 * fp32 summation order (that entry point splits K over CTAs when the output
 * tiles are few, and from M = 17 runs the tensor-core GEMM). */
int w4_gptq_gemm_fp8_noalloc(const void *a, int a_dtype, const int32_t *qweight,
                             const int32_t *qzeros, const uint16_t *scales, uint8_t *q_out,
                             float *row_scale, int M, int N, int K, int group_size,
                             int zero_offset, void *stream);

/* Grouped (MoE) GEMMs: one launch over num_experts experts (1..64).  Expert e's weights are
 * slice e of stacked tensors and its tokens are rows [offsets[e], offsets[e+1]) of a and c
 * (host array of num_experts + 1 ints, offsets[0] == 0, nondecreasing; tokens sorted by
 * expert; empty experts allowed).  The reference runs the routed experts of a MoE layer as
 * separate GEMMs chained on one queue (kernels/esimd_dpas/moe_group_s8_m1.cpp:1-7; expert shapes
 * hidden 2688, expert 1856, kernels/nemotron/README.md).  The decode GEMM streams each expert's
 * weights once per 16 tokens of that expert, so it is meant for decode-sized groups.
 * GPTQ: qweight [E][K/8][N], qzeros [E][K/gs][N/8] or NULL, scales [E][K/gs][N]; arguments
 * otherwise as w4_gptq_gemm (no act_order).  c_dtype f16, bf16, f32 or e4m3 (row_scale then
 * holds one scale per row of c).  The workspace follows the rules of w4_gptq_gemm. */
size_t w4_gptq_gemm_grouped_workspace_bytes(const int32_t *offsets, int num_experts, int N, int K,
                                            int group_size, int c_dtype);
int w4_gptq_gemm_grouped(const void *a, int a_dtype, const int32_t *qweight, const int32_t *qzeros,
                         const uint16_t *scales, const int32_t *offsets, int num_experts, void *c,
                         int c_dtype, float *row_scale, int N, int K, int group_size, int zero_offset,
                         void *workspace, size_t workspace_bytes, void *stream);
/* NVFP4 W4A16: w [E][N][K/2] (K-contiguous codes), E4M3 block scales [E][K/16][N], tensor scales
 * global_scale[E] (fp32, device), bf16 activations; K a multiple of 64, N of 32. */
size_t w4_nvfp4_gemm_grouped_workspace_bytes(const int32_t *offsets, int num_experts, int N, int K,
                                             int c_dtype);
int w4_nvfp4_gemm_grouped(const void *a, const uint8_t *w, const uint8_t *scale, const float *global_scale,
                          const int32_t *offsets, int num_experts, void *c, int c_dtype, float *row_scale,
                          int N, int K, void *workspace, size_t workspace_bytes, void *stream);

/* The reference kernel's own contract, same arguments in the same order as
 * launch(q, ad, bd, asd, sd, cd, rows, cols, dk) of
 * kernels/esimd_dpas/dpas_s4_gptq_sc.cpp:146-149:
 *   C[r,c] = half( sum_g float(s32_g) * a_scale[r] * float(b_scale[g,c]) ),
 *   s32_g  = sum_{k in g} A_s4[r,k] * B_s4[k,c]   (group size 128, exact)
 * a_s4 u8 [rows, dk/2] (pack_a, low nibble = even k), b_s4 u8 [dk/2, cols]
 * (pack_b), a_scale f32 [rows], b_scale f16 [dk/128, cols], c f16 [rows, cols].
 * Bit-exact with the reference host oracle (dpas_s4_gptq_sc.cpp:273-288). */
int w4_gptq_gemm_s4a(const uint8_t *a_s4, const uint8_t *b_s4, const float *a_scale,
                     const uint16_t *b_scale, uint16_t *c, int rows, int cols, int dk,
                     void *stream);

/* ===================================================================== */
/* NVFP4                                                                  */
/* ===================================================================== */

/* Dequantise to fp32, bit-exact: w[k,n] = (e2m1(nib[k,n]) * s[k/16,n]) * global.
 * scale: [K/16,N] of scale_dtype W4_E4M3 (then global_scale is an f32[1] device
 * pointer) or W4_BF16 (folded scale; global_scale must be NULL).
 * Replaces unpack_host of kernels/nvfp4/nibble_lut_sc.cpp:85-92 with the block
 * scales of the external op (kernels/nvfp4/bench_nvfp4_m1.py:84-88). */
int w4_nvfp4_dequant(const uint8_t *w, int layout, const void *scale, int scale_dtype,
                     const float *global_scale, int K, int N, float *out, void *stream);

/* Quantise bf16 activations to NVFP4, bit-exact with the host definition:
 *   sf = e4m3(amax16 / (6 * a_global)),  d = e4m3(sf) * a_global,
 *   code = e2m1(a * (1 / d))   (one correctly rounded reciprocal per block)
 * a: bf16 [M,K]; a_global: f32[1] device pointer (the tensor decode scale);
 * codes u8 [M,K/2] (low nibble = even k); sf u8 [M,K/16]. */
int w4_nvfp4_quant_act(const uint16_t *a, int M, int K, const float *a_global,
                       uint8_t *codes, uint8_t *sf, void *stream);

size_t w4_nvfp4_workspace_bytes(int M, int N, int K, int act_mode, int c_dtype);

/* NVFP4 GEMM:  C[m,n] = (sum_k A[m,k] * (e2m1(w[k,n]) * s[k/16,n])) * global
 * a: bf16 [M,K]; w, layout, scale, scale_dtype, global_scale as in
 * w4_nvfp4_dequant; act_mode W4_ACT_W4A16 (a used as is) or W4_ACT_NVFP4 (a
 * quantised per w4_nvfp4_quant_act with a_global first; needs workspace);
 * c, c_dtype, row_scale as in w4_gptq_gemm.  Weights must be in the W4_NVFP4_NK
 * layout (w4_nvfp4_repack_kn_to_nk converts the other).  Shapes: K % 128 == 0,
 * N % 32 == 0, M >= 1.
 * Replaces the external op nvfp4_gemm_w4a16(x, w, None, scale, 16) /
 * nvfp4_gemm_w4a16_f8scale(x, w, None, bscale, gscale, 16)
 * (kernels/nvfp4/bench_nvfp4_m1.py:67,88) and launch() of
 * kernels/nvfp4/nibble_lut_sc.cpp:198-290. */
int w4_nvfp4_gemm(const void *a, const uint8_t *w, int layout, const void *scale,
                  int scale_dtype, const float *global_scale, int act_mode,
                  const float *a_global, void *c, int c_dtype, float *row_scale, int M, int N,
                  int K, void *workspace, size_t workspace_bytes, void *stream);

/* Load-time transpose of packed weights from the reference kernel's layout
 * u8 [K/2, N] (kernels/nvfp4/nibble_lut_sc.cpp:77-83) to the K-contiguous
 * u8 [N, K/2] that w4_nvfp4_gemm reads.  Block scales keep their [K/16, N]
 * layout.  w_nk must not alias w_kn. */
int w4_nvfp4_repack_kn_to_nk(const uint8_t *w_kn, int K, int N, uint8_t *w_nk, void *stream);

/* Load-time rearrangement of E4M3 block scales [K/16, N] into the layout the
 * block-scaled tensor-core GEMM reads (act_mode W4_ACT_NVFP4): 512-byte atoms of
 * 128 columns x 4 blocks, byte (n % 32) * 16 + (n / 32 % 4) * 4 + (kb % 4), atoms
 * ordered [n / 128][kb / 4]; N rounded up to 128 with zero scales.  Size
 * w4_nvfp4_scale_atoms_bytes(N, K).  Pass the result to w4_nvfp4_gemm with
 * scale_dtype W4_E4M3_ATOMS (the per-call rearrangement is then skipped).
 * No counterpart in the reference (its NVFP4 operator is external). */
size_t w4_nvfp4_scale_atoms_bytes(int N, int K);
int w4_nvfp4_repack_scales(const uint8_t *scale, int K, int N, uint8_t *atoms, void *stream);

/* Producer fusion (RMSNorm -> NVFP4 activations) and the GEMM that consumes it.
 *
 * w4_rmsnorm_quant_nvfp4: one pass per row of x f16/bf16 [M,K] (x_dtype):
 *   inv = 1 / sqrt(sum_k x^2 / K + eps),  y = bf16(x * inv [* gamma])
 * then y quantised exactly as w4_nvfp4_quant_act does, with the codes written
 * to codes u8 [rows, K/2] and the block scales to sf_atoms in the 512-byte atom
 * layout of the block-scaled GEMM, rows = M rounded up to 128 (the padding
 * rows get zero codes and scales).  gamma: [K] of x_dtype or NULL (none).
 * Buffer sizes: w4_nvfp4_act_codes_bytes(M, K), w4_nvfp4_scale_atoms_bytes(M, K).
 * K % 64 == 0.  The normalisation is the reference's contract
 * (kernels/epilogue_quant/rmsnorm_epilogue.cpp:39-56); the reference follows it
 * with an s8 cast (w4_rmsnorm_quant_s8) in a second kernel or fused
 * (:118-151); the fused NVFP4 producer is the next step its K5 summary names
 * (results/k5/SUMMARY.md:65-80).
 *
 * w4_nvfp4_gemm_q: w4_nvfp4_gemm with act_mode W4_ACT_NVFP4 for activations
 * already quantised (codes + scale atoms as written above, a_global the
 * tensor scale they were quantised with).  Same weights, outputs and shape
 * rules (K % 256 == 0, N % 128 == 0, E4M3 or E4M3-atom weight scales);
 * workspace from w4_nvfp4_gemm_q_workspace_bytes. */
size_t w4_nvfp4_act_codes_bytes(int M, int K);
int w4_rmsnorm_quant_nvfp4(const void *x, int x_dtype, const void *gamma, float eps, const float *a_global,
                           uint8_t *codes, uint8_t *sf_atoms, int M, int K, void *stream);
size_t w4_nvfp4_gemm_q_workspace_bytes(int M, int N, int K, int scale_dtype, int c_dtype);
int w4_nvfp4_gemm_q(const uint8_t *a_codes, const uint8_t *a_sf_atoms, const float *a_global, const uint8_t *w,
                    int layout, const void *scale, int scale_dtype, const float *global_scale, void *c,
                    int c_dtype, float *row_scale, int M, int N, int K, void *workspace, size_t workspace_bytes,
                    void *stream);

/* The reference LUT kernel's own contract, same arguments in the same order as
 * launch(q, ad, pd, asd, bsd, cd, rows, cols, dk) of
 * kernels/nvfp4/nibble_lut_sc.cpp:198-201:
 *   C[r,c] = half( (sum_k A_s8[r,k] * q[k,c]) * a_s[r] * b_s[c] ),  q = 2*e2m1
 * a s8 [rows, dk], packed u8 [dk/2, cols], a_s f32 [rows], b_s f32 [cols],
 * c f16 [rows, cols].  Bit-exact with nibble_lut_sc.cpp:319-330. */
int w4_nvfp4_lut_gemm_s8a(const int8_t *a, const uint8_t *packed, const float *a_s,
                          const float *b_s, uint16_t *c, int rows, int cols, int dk,
                          void *stream);

/* ===================================================================== */
/* epilogue quant                                                         */
/* ===================================================================== */

/* Fused RMSNorm (gamma = 1) + symmetric per-row s8 quantisation:
 *   inv = 1/sqrt(mean(x^2) + eps); y = x*inv; s = max|y|/127 (1 if 0);
 *   q = clamp(rint(y/s), -127, 127)
 * x f16 [M,K], q s8 [M,K], scale f32 [M].  Same arguments as launch_fused(q, x,
 * q, s, m, k) of kernels/epilogue_quant/rmsnorm_epilogue.cpp:118-119 plus eps
 * (the reference fixes 1e-6, :23). */
int w4_rmsnorm_quant_s8(const uint16_t *x, int8_t *q, float *scale, int M, int K, float eps,
                        void *stream);

/* Per-row fp8-E4M3 cast of a finished [M,N] tensor (f16 / bf16 / f32):
 * s = max|y_row|/448 (1 if 0), q = e4m3_rne_satfinite(y/s).  The same cast
 * the GEMMs apply in their epilogue when c_dtype == W4_E4M3. */
int w4_rowscale_fp8(const void *y, int y_dtype, uint8_t *q, float *row_scale, int M, int N,
                    void *stream);

/* ===================================================================== */
/* tensor parallelism                                                     */
/* ===================================================================== */

/* One process per GPU.  Column-parallel layers (QKV, gate|up) hold N/TP output
 * columns of every sub-matrix and need no exchange; row-parallel layers (o,
 * down) hold K/TP input rows (whole groups) and sum their partial [M,N]
 * outputs with an NCCL all-reduce over NVLink.  The reference's counterpart is
 * the collective alone: an in-place bf16 all_reduce(SUM) over torch's xccl
 * backend (parallel/tp2/bench_xccl_p2p0.py:235-251). */
typedef struct w4_tp_comm w4_tp_comm;

enum w4_tp_mode {
    W4_TP_COLUMN = 0,
    W4_TP_ROW = 1
};

#define W4_TP_UNIQUE_ID_BYTES 128

/* Rank 0 creates the id (host buffer of W4_TP_UNIQUE_ID_BYTES) and the host
 * hands it to every rank by its own means (a store, MPI, a file). */
int w4_tp_get_unique_id(uint8_t *id);

/* Join the communicator of `nranks` ranks as `rank`, on the current CUDA
 * device.  Returns W4_ERR_TIMEOUT (and creates nothing) when the other ranks
 * have not joined within timeout_ms. */
int w4_tp_comm_init(w4_tp_comm **comm, int nranks, int rank, const uint8_t *id, int timeout_ms);
int w4_tp_comm_destroy(w4_tp_comm *comm);
/* Tear down without waiting for the other ranks (after a failure on any rank). */
int w4_tp_comm_abort(w4_tp_comm *comm);

/* In-place sum over all ranks of buf[count] (f16 / bf16 / f32), enqueued on stream. */
int w4_tp_allreduce(w4_tp_comm *comm, void *buf, size_t count, int dtype, void *stream);

/* Wait (host side) until everything enqueued on stream is done.  If it is not
 * done within timeout_ms (a peer never reached the collective) or NCCL reports
 * an error, the communicator is aborted and W4_ERR_TIMEOUT / W4_ERR_NCCL is
 * returned; an aborted communicator refuses further calls. */
int w4_tp_wait(w4_tp_comm *comm, void *stream, int timeout_ms);

/* on = 1: row-parallel decode layers (M <= 16, no act_order permutation, peer
 * memory mapped between the ranks) run one fused kernel: each CTA pushes its
 * fp32 partial tile to every rank over NVLink, waits (bounded) for the same
 * tile of every other rank and stores the rank-ordered sum, with no separate
 * all-reduce launch.  on = 0 (the default): GEMM + w4_tp_allreduce, which
 * measures faster on B200 pairs so far.  Every rank must choose the same.  The
 * reference has no fused form; its TP step is a bare all-reduce
 * (parallel/tp2/bench_xccl_p2p0.py:235-251). */
int w4_tp_set_fused_epilogue(w4_tp_comm *comm, int on);

size_t w4_tp_linear_workspace_bytes(int mode, int M, int N, int K, int group_size, int has_perm,
                                    int c_dtype);

/* One GPTQ linear shard.  Arguments as w4_gptq_gemm on this rank's shard:
 *   W4_TP_COLUMN: qweight [K/8, N_rank] etc.; c [M, N_rank]; comm may be NULL.
 *   W4_TP_ROW:    a [M, K_rank], qweight [K_rank/8, N], K_rank a multiple of
 *                 group_size; c [M, N] receives the sum over ranks.  With
 *                 c_dtype W4_E4M3 the sum is taken in f32 (workspace) and then
 *                 cast with its per-row scale. */
int w4_tp_linear(w4_tp_comm *comm, int mode, const void *a, int a_dtype, const int32_t *qweight,
                 const int32_t *qzeros, const uint16_t *scales, const int32_t *perm, void *c,
                 int c_dtype, float *row_scale, int M, int N, int K, int group_size,
                 int zero_offset, void *workspace, size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* W4_H */
