/*
 * qgemv_b200.h -- C-ABI of the B200 (sm_100a) quantized decode GEMV library
 * (libqgemv_b200.so).
 *
 * Two groups of entry points:
 *
 *  1. Drop-in launchers.  Same names, argument lists, argument meaning and error
 *     behaviour as the reference's `extern "C"` launchers in
 *     runtime/kernels/decode/decode_kernels.h (cited per declaration).  An app of
 *     the reference links this library instead of decode_kernels.cu and runs
 *     unchanged: logits for the launched rows, the KV page write with the
 *     pre-update token, then token = (argmax + token + 1) % 32000.
 *
 *  2. New entry points (prefix qg_): pure GEMV over any of the eight pack formats,
 *     batch > 1, the fused layer-slice epilogues, dequantize-to-fp32, and the
 *     error word.  They have no counterpart in the reference unless a citation
 *     says so.
 *
 * Every pointer is caller-owned device memory unless stated otherwise.  No launching
 * entry point allocates, synchronizes or touches host memory, so all of them can be
 * recorded into a CUDA graph; the exceptions are qg_get_error (reads the error word)
 * and the qg_graph_* functions (they build and own a graph).  Errors: invalid
 * arguments return cudaErrorInvalidValue before any launch; otherwise the result of
 * cudaGetLastError() after the launches.
 */
#ifndef QGEMV_B200_H_
#define QGEMV_B200_H_

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------------------
 * Pack formats.  Byte layouts are the reference's resident packs:
 *   Q4K_RAW            144 B GGUF blocks {f16 d, f16 dmin, u8 scales[12], u8 qs[128]}
 *                      (decode_kernels.cu:1920-2001)
 *   Q4K_SPLIT_*        payload stream 128 B/blk (= block[16:144]) plus a metadata
 *                      stream (tools/bench/q4k_resident_pack.py:82-145):
 *     PREDECODED       64 B/blk: 8 x {f32 d*scale, f32 dmin*min}
 *     HALF             32 B/blk: 8 x {f16 d*scale, f16 dmin*min}
 *     COMPACT          20 B/blk: {f16 d, f16 dmin, u8 scale[8], u8 min[8]}
 *     NATIVE           16 B/blk: block[0:16]
 *   Q5K                176 B {f16 d, f16 dmin, scales[12], qh[32], qs[128]}
 *   IQ2S               82 B  {f16 d, qs[64], qh[8], scales[8]}
 *   IQ3S               110 B {f16 d, qs[64], qh[8], signs[32], scales[4]}
 * Each block holds 256 consecutive values of one row; a row of `cols` values is
 * cols/256 consecutive blocks; rows are stored one after another.
 * ------------------------------------------------------------------------- */
typedef enum qg_format {
  QG_FMT_Q4K_RAW = 0,
  QG_FMT_Q4K_SPLIT_PREDECODED = 1,
  QG_FMT_Q4K_SPLIT_HALF = 2,
  QG_FMT_Q4K_SPLIT_COMPACT = 3,
  QG_FMT_Q4K_SPLIT_NATIVE = 4,
  QG_FMT_Q5K = 5,
  QG_FMT_IQ2S = 6,
  QG_FMT_IQ3S = 7,
  QG_FMT_COUNT = 8
} qg_format;

/* Bytes per 256-value block in the payload stream. */
static inline uint32_t qg_payload_bytes_per_block(int fmt) {
  switch (fmt) {
    case QG_FMT_Q4K_RAW: return 144u;
    case QG_FMT_Q4K_SPLIT_PREDECODED:
    case QG_FMT_Q4K_SPLIT_HALF:
    case QG_FMT_Q4K_SPLIT_COMPACT:
    case QG_FMT_Q4K_SPLIT_NATIVE: return 128u;
    case QG_FMT_Q5K: return 176u;
    case QG_FMT_IQ2S: return 82u;
    case QG_FMT_IQ3S: return 110u;
    default: return 0u;
  }
}

/* Bytes per 256-value block in the metadata stream (0 = no metadata stream). */
static inline uint32_t qg_meta_bytes_per_block(int fmt) {
  switch (fmt) {
    case QG_FMT_Q4K_SPLIT_PREDECODED: return 64u;
    case QG_FMT_Q4K_SPLIT_HALF: return 32u;
    case QG_FMT_Q4K_SPLIT_COMPACT: return 20u;
    case QG_FMT_Q4K_SPLIT_NATIVE: return 16u;
    default: return 0u;
  }
}

/* Error word bits (set by kernels, read and cleared by qg_get_error). */
#define QG_ERR_WAIT_TIMEOUT 0x1u /* a bounded wait (TMA barrier, exchange word) ran out */
#define QG_ERR_POSITION 0x2u     /* a decode position read from device memory was past the
                                    KV cache or the step graph's context bucket */

/* ===========================================================================
 * 1. Drop-in launchers (reference: runtime/kernels/decode/decode_kernels.h)
 * ========================================================================= */

/* decode_kernels.h:424-435 (raw 144-B Q4_K blocks; all rows). */
cudaError_t rtxllm_launch_q4k_matvec_decode(
    const uint8_t* q4k_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:437-448 */
cudaError_t rtxllm_launch_q4k_matvec_decode_shared(
    const uint8_t* q4k_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:450-461 */
cudaError_t rtxllm_launch_q4k_matvec_decode_warp(
    const uint8_t* q4k_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:463-474 */
cudaError_t rtxllm_launch_q4k_matvec_decode_warp_broadcast(
    const uint8_t* q4k_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:476-487 */
cudaError_t rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4(
    const uint8_t* q4k_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:489-500 */
cudaError_t rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x2(
    const uint8_t* q4k_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:502-513 */
cudaError_t rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x4(
    const uint8_t* q4k_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:515-527.  The (scale*d, min*dmin) side table is accepted for
 * signature compatibility; the raw blocks already carry the same information. */
cudaError_t rtxllm_launch_q4k_matvec_decode_predecoded_vec4x4(
    const uint8_t* q4k_blocks, const float* q4k_scale_min_pairs, const float* activation,
    float* logits, float* kv, uint32_t* token, uint32_t rows, uint32_t cols,
    uint32_t kv_words, uint32_t page_words, uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:529-541 */
cudaError_t rtxllm_launch_q4k_matvec_decode_split_predecoded_vec4x4(
    const uint8_t* q4k_payload, const float* q4k_scale_min_pairs, const float* activation,
    float* logits, float* kv, uint32_t* token, uint32_t rows, uint32_t cols,
    uint32_t kv_words, uint32_t page_words, uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:543-555 */
cudaError_t rtxllm_launch_q4k_matvec_decode_split_half_vec4x4(
    const uint8_t* q4k_payload, const uint16_t* q4k_scale_min_half_pairs,
    const float* activation, float* logits, float* kv, uint32_t* token, uint32_t rows,
    uint32_t cols, uint32_t kv_words, uint32_t page_words, uint32_t active_pages,
    cudaStream_t stream);
/* decode_kernels.h:557-569 */
cudaError_t rtxllm_launch_q4k_matvec_decode_split_compact_vec4x4(
    const uint8_t* q4k_payload, const uint8_t* q4k_compact_meta, const float* activation,
    float* logits, float* kv, uint32_t* token, uint32_t rows, uint32_t cols,
    uint32_t kv_words, uint32_t page_words, uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:571-583 */
cudaError_t rtxllm_launch_q4k_matvec_decode_split_native_vec4x4(
    const uint8_t* q4k_payload, const uint8_t* q4k_native_meta, const float* activation,
    float* logits, float* kv, uint32_t* token, uint32_t rows, uint32_t cols,
    uint32_t kv_words, uint32_t page_words, uint32_t active_pages, cudaStream_t stream);

/* decode_kernels.h:345-357.  Rows [0, min(rows, rows_limit)) only. */
cudaError_t rtxllm_launch_q5k_matvec_decode_probe(
    const uint8_t* q5k_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t rows_limit, uint32_t kv_words,
    uint32_t page_words, uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:359-366 (logits only: no KV write, no token update). */
cudaError_t rtxllm_launch_iq2s_matvec_probe(
    const uint8_t* iq2s_blocks, const float* activation, float* logits, uint32_t rows,
    uint32_t cols, uint32_t rows_limit, cudaStream_t stream);
/* decode_kernels.h:368-380 */
cudaError_t rtxllm_launch_iq2s_matvec_decode_probe(
    const uint8_t* iq2s_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t rows_limit, uint32_t kv_words,
    uint32_t page_words, uint32_t active_pages, cudaStream_t stream);
/* decode_kernels.h:382-394 */
cudaError_t rtxllm_launch_iq3s_matvec_decode_probe(
    const uint8_t* iq3s_blocks, const float* activation, float* logits, float* kv,
    uint32_t* token, uint32_t rows, uint32_t cols, uint32_t rows_limit, uint32_t kv_words,
    uint32_t page_words, uint32_t active_pages, cudaStream_t stream);

/* decode_kernels.h:319-325: token = (argmax(logits[0:rows]) + token_offset) % vocab_size. */
cudaError_t rtxllm_launch_output_token_sample(
    const float* logits, uint32_t* token, uint32_t rows, uint32_t vocab_size,
    uint32_t token_offset, cudaStream_t stream);

/* Feedback kernels of the mixed layer-slice runner (decode_kernels.h:38-101).  All use
 * the unweighted RMS of logits[0:rows] and index logits[col % rows]. */
cudaError_t rtxllm_launch_rmsnorm_feedback(
    const float* logits, float* activation, uint32_t rows, uint32_t cols, float epsilon,
    cudaStream_t stream);
cudaError_t rtxllm_launch_silu_rmsnorm_feedback(
    const float* logits, float* activation, uint32_t rows, uint32_t cols, float epsilon,
    cudaStream_t stream);
cudaError_t rtxllm_launch_rmsnorm_feedback_with_silu_cache(
    const float* logits, float* activation, float* silu_cache, uint32_t rows, uint32_t cols,
    float epsilon, cudaStream_t stream);
cudaError_t rtxllm_launch_gated_silu_rmsnorm_feedback(
    const float* logits, const float* silu_cache, float* activation, uint32_t rows,
    uint32_t cache_cols, uint32_t cols, float epsilon, cudaStream_t stream);
cudaError_t rtxllm_launch_rmsnorm_silu_cache(
    const float* logits, float* silu_cache, uint32_t rows, uint32_t cache_cols, float epsilon,
    uint32_t accumulate, cudaStream_t stream);
cudaError_t rtxllm_launch_rmsnorm_cache(
    const float* logits, float* cache, uint32_t rows, uint32_t cache_cols, float epsilon,
    uint32_t accumulate, cudaStream_t stream);
cudaError_t rtxllm_launch_rmsnorm_cache_and_gated_product(
    const float* logits, const float* gate_cache, float* up_cache, float* activation,
    uint32_t rows, uint32_t cache_cols, uint32_t output_cols, float epsilon,
    uint32_t accumulate, cudaStream_t stream);

/* ===========================================================================
 * 2. New entry points
 * ========================================================================= */

/* y[r] = sum_c W[r, c] * x[c] for r < rows.  `meta` is the metadata stream for the
 * Q4K_SPLIT_* formats and ignored otherwise.  cols must be a positive multiple of
 * 256.  No KV write, no token update. */
cudaError_t qg_gemv(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                    float* y, uint32_t rows, uint32_t cols, cudaStream_t stream);

/* Prepared activations.  Every GEMV CTA needs x as two int8 planes per 32 columns
 * (x ~= s * (hi + lo / 256), |error| <= 3.2e-5 * ||x||_inf).  qg_act_prepare computes
 * them once into `act` (qg_act_bytes(cols) bytes, 16-B aligned, caller-owned) so the
 * GEMVs that read the same x skip that work; qg_gemv does it inside the kernel. */
cudaError_t qg_act_bytes(uint32_t cols, size_t* bytes);
cudaError_t qg_act_prepare(const float* x, uint32_t cols, void* act, cudaStream_t stream);

/* qg_gemv reading x through a prepared activation of the same x (act may be NULL). */
cudaError_t qg_gemv_act(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                        const void* act, float* y, uint32_t rows, uint32_t cols,
                        cudaStream_t stream);

/* One decode stage with the reference launchers' semantics (decode_kernels.cu:
 * 4032-4177): y for rows [0, rows), KV page write with the pre-update token for
 * rows < active_pages (kv may be NULL), then
 * token = (argmax(y[0:rows]) + token + 1) % 32000. */
cudaError_t qg_decode_stage(int fmt, const uint8_t* payload, const uint8_t* meta,
                            const float* x, float* y, float* kv, uint32_t* token,
                            uint32_t rows, uint32_t cols, uint32_t kv_words,
                            uint32_t page_words, uint32_t active_pages, cudaStream_t stream);

/* Y[b, r] = sum_c W[r, c] * X[b, c] for b < batch (X row-major [batch, cols] fp32,
 * Y row-major [batch, rows]).  batch 1..32, every format.  On the CUDA cores: each group
 * of up to 8 vectors is one pass over the weights (multi-vector GEMV, csrc/qg_gemv_batch.cu:
 * x as int16 with one scale per vector and column slice, |error| <= 1.6e-5 *
 * ||w_row||_1 * ||x_b||_inf plus fp32 rounding; deterministic); a single vector takes the
 * batch-1 GEMV.  Packs whose payload or metadata is not 16-B aligned go vector by vector. */
cudaError_t qg_gemv_batched(int fmt, const uint8_t* payload, const uint8_t* meta,
                            const float* x, float* y, uint32_t batch, uint32_t rows,
                            uint32_t cols, cudaStream_t stream);

/* Dequantize blocks [first_block, first_block + block_count) of a pack into
 * out[block_count * 256] (fp32, bit-identical to the reference's CPU decode). */
cudaError_t qg_dequantize(int fmt, const uint8_t* payload, const uint8_t* meta,
                          uint64_t first_block, uint64_t block_count, float* out,
                          cudaStream_t stream);

/* token = (argmax(values[0:n]) + token_offset + add_token * token) % modulus, the
 * lowest index winning ties (argmax_token_kernel / output_token_sample_kernel,
 * decode_kernels.cu:2993-3073).  add_token = 1, token_offset = 1, modulus = 32000
 * reproduces the launchers' token update. */
cudaError_t qg_argmax_token(const float* values, uint32_t n, uint32_t* token,
                            uint32_t token_offset, uint32_t add_token, uint32_t modulus,
                            cudaStream_t stream);

/* Batched decode GEMM (no reference counterpart -- every reference matvec kernel is
 * batch 1): Y[b, r] = sum_c W[r, c] * X[b, c] for b < batch, X row-major [batch, cols]
 * fp32, Y row-major [batch, rows] fp32, batch 1..32.  Below batch 5 it runs the CUDA-core
 * multi-vector GEMV of qg_gemv_batched (workspace unused); from batch 5 the tensor cores
 * (the crossover measured on B200; the QG_TC_MIN_BATCH environment variable, 2..33, moves it):
 * Formats: QG_FMT_Q4K_RAW, QG_FMT_Q5K, QG_FMT_IQ2S, QG_FMT_IQ3S (payload 16-B aligned;
 * `meta` unused).  Weights are expanded to exact fp16 integer tiles and contracted
 * with tcgen05.mma (M=128, N=16 or 32) against x scaled by a power of two per batch row
 * and rounded to fp16; |error| <= 2^-11 * ||w_row||_1 * ||x_b||_inf.  Results are
 * deterministic.  Three launches on `stream`; `workspace` (256-B aligned, caller-owned) holds the
 * prepared x and the split-row partial sums: qg_gemm_batched_workspace_bytes (sized for
 * grids of up to 256 CTAs, so the size does not depend on the device it is queried on). */
cudaError_t qg_gemm_batched_workspace_bytes(int fmt, uint32_t batch, uint32_t rows, uint32_t cols,
                                            size_t* bytes);
cudaError_t qg_gemm_batched(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                            float* y, uint32_t batch, uint32_t rows, uint32_t cols, void* workspace,
                            cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * Mixed-format layer slice (no reference counterpart for the
 * weighted RMSNorm, the SiLU gate or the residual add -- the reference's slice uses
 * unweighted feedback kernels and a passthrough attention phase,
 * runtime/apps/mixed_sequence_benchmark_runner/main.cpp:195,4073-4280):
 *   h = x / sqrt(mean(x^2) + eps) * norm_weight
 *   q = Wq h,  k = Wk h,  v = Wv h           (attn_fmt; Wq [q_rows x hidden],
 *                                              Wk/Wv [kv_rows x hidden])
 *   o = Wo q                                 (attention passthrough; Wo [hidden x q_rows])
 *   a = silu(Wg o) * (Wu o)                  (ffn_fmt; Wg/Wu [ffn x hidden])
 *   out = x + Wd a                           (down_fmt; Wd [hidden x ffn])
 * Eight kernel launches on `stream` (see csrc/qg_slice.cu); intermediates live in a
 * caller-owned workspace of qg_layer_slice_workspace_bytes() bytes (256-B aligned).
 * ------------------------------------------------------------------------- */
typedef struct qg_layer_slice {
  uint32_t hidden, q_rows, kv_rows, ffn;
  float eps;
  const float* norm_weight;
  int attn_fmt;
  const uint8_t *wq, *wk, *wv, *wo;
  const uint8_t *wq_meta, *wk_meta, *wv_meta, *wo_meta;
  int ffn_fmt;
  const uint8_t *wg, *wu;
  const uint8_t *wg_meta, *wu_meta;
  int down_fmt;
  const uint8_t* wd;
  const uint8_t* wd_meta;
} qg_layer_slice;

/* Device pointers of the slice's intermediate vectors inside a workspace. */
typedef struct qg_layer_slice_views {
  float *h, *q, *k, *v, *o, *gate, *up, *act;
} qg_layer_slice_views;

cudaError_t qg_layer_slice_workspace_bytes(const qg_layer_slice* s, size_t* bytes);
cudaError_t qg_layer_slice_buffers(const qg_layer_slice* s, void* workspace,
                                   qg_layer_slice_views* views);
cudaError_t qg_layer_slice_forward(const qg_layer_slice* s, const float* x, float* out,
                                   void* workspace, cudaStream_t stream);

/* Workspace-free form of qg_layer_slice_forward (no reference counterpart: the
 * reference's runner always owns its device buffers).  For callers that cannot
 * allocate device memory -- a plugin host that hands over only weights, activations
 * and a stream; a serving process whose allocator already holds nearly all of HBM;
 * a decode loop where cudaMalloc/cudaFree would synchronise the device.  The slice's
 * intermediates live in a library-owned device array of QG_SLICE_STATIC_SCRATCH_BYTES
 * per device (enough for hidden 8192 / ffn 28672); nothing is allocated or freed.
 *  - Returns cudaErrorInvalidValue when qg_layer_slice_workspace_bytes(s) exceeds
 *    QG_SLICE_STATIC_SCRATCH_BYTES (use qg_layer_slice_forward with a workspace).
 *  - The array's device address belongs to one CUDA context.  The first call in each
 *    context (the first on each device, the first after cudaDeviceReset, the first
 *    under another driver-API context) looks it up (cudaGetSymbolAddress) and caches
 *    it with the context's id; make that first call before any stream capture.
 *  - One array per device: calls whose work overlaps on a device (different streams
 *    or host threads) race on it; serialise them on one stream. */
#define QG_SLICE_STATIC_SCRATCH_BYTES (1u << 20)
cudaError_t qg_layer_slice_forward_static(const qg_layer_slice* s, const float* x, float* out,
                                          cudaStream_t stream);

/* Decode-step graphs (runtime/apps/mixed_sequence_benchmark_runner/main.cpp:4801-4823
 * captures, instantiates and uploads one graph, then replays it): everything enqueued
 * on `stream` between qg_graph_begin and qg_graph_end becomes one graph; the handle
 * owns it until qg_graph_destroy. */
typedef struct qg_graph_s* qg_graph;
cudaError_t qg_graph_begin(cudaStream_t stream);
cudaError_t qg_graph_end(cudaStream_t stream, qg_graph* out);
cudaError_t qg_graph_launch(qg_graph graph, cudaStream_t stream);
cudaError_t qg_graph_destroy(qg_graph graph);

/* The layer slice for `batch` hidden vectors at once (x, out row-major [batch][hidden],
 * batch 1..32): the same stages as qg_layer_slice_forward -- per-row RMSNorm (the same
 * sum-of-squares order, so each row's h matches the single-vector slice bit for bit),
 * Q/K/V/O, gate/up, SiLU-gate, down, residual -- with every GEMV a batched one routed
 * like qg_gemm_batched (CUDA-core multi-vector GEMV below the tensor-core threshold,
 * tcgen05 tiles above it for the GGUF formats); batch 1 is qg_layer_slice_forward
 * itself.  Activations per GEMV as in
 * qg_gemv_batched / qg_gemm_batched.  Workspace: qg_layer_slice_batched_workspace_bytes
 * (256-B aligned); views into it: qg_layer_slice_batched_buffers ([batch][n] each). */
cudaError_t qg_layer_slice_batched_workspace_bytes(const qg_layer_slice* s, uint32_t batch,
                                                   size_t* bytes);
cudaError_t qg_layer_slice_forward_batched(const qg_layer_slice* s, const float* x, float* out,
                                           uint32_t batch, void* workspace, cudaStream_t stream);
cudaError_t qg_layer_slice_batched_buffers(const qg_layer_slice* s, uint32_t batch, void* workspace,
                                           qg_layer_slice_views* views);

/* One captured graph per decode step and batch bucket (the reference's
 * CudaGraphBucketDescriptor.batch_bucket, runtime/core/graphs/cuda_graph_bucket.h:16-23,
 * whose graphs the reference never builds): qg_slice_buckets_create waits for the work
 * pending on `stream` (any stream, the legacy default one included), then captures
 * qg_layer_slice_forward_batched once per bucket (`batches` ascending, 1..32, at most 32
 * buckets) on a stream of its own and returns when the graphs are uploaded; each bucket
 * owns its padded input/output rows and workspace, allocated here.
 * qg_slice_buckets_run(x, out, batch) uses the smallest bucket >= batch: the batch's rows
 * are copied in, the bucket's graph replayed and the rows copied out (two device copies
 * and one graph launch on `stream`; cudaErrorInvalidValue past the largest bucket).  Rows
 * past `batch` never affect the live rows.  Runs of one handle must not overlap. */
typedef struct qg_slice_buckets_s* qg_slice_buckets;
cudaError_t qg_slice_buckets_create(const qg_layer_slice* s, const uint32_t* batches, uint32_t n,
                                    cudaStream_t stream, qg_slice_buckets* out);
cudaError_t qg_slice_buckets_bucket(qg_slice_buckets b, uint32_t batch, uint32_t* bucket);
cudaError_t qg_slice_buckets_run(qg_slice_buckets b, const float* x, float* out, uint32_t batch,
                                 cudaStream_t stream);
cudaError_t qg_slice_buckets_destroy(qg_slice_buckets b);

/* ---------------------------------------------------------------------------
 * Tensor-parallel decode step of a Llama-style mixed-quant model (
 * no reference counterpart -- the reference is single-GPU with synthetic attention).
 * One process per GPU.  Rank r of tp_size holds row shards of Wq/Wk/Wv (its
 * n_q_heads/tp and n_kv_heads/tp heads), Wg/Wu (ffn/tp rows) and the vocab head
 * (qg_decoder_shard gives its rows and offset), column shards of Wo (its q heads'
 * columns) and Wd (its ffn/tp columns), and its kv heads' fp16 KV cache
 * [n_kv_heads/tp][ctx_max][head_dim].  Per layer: rmsnorm -> q,k,v -> RoPE (adjacent
 * pairs, angle pos * rope_base^(-2i/head_dim)) and cache append at `pos` -> GQA
 * attention over positions [0, pos] -> Wo -> all-reduce (+x) -> rmsnorm -> gate,up ->
 * silu(g)*u -> Wd -> all-reduce (+x1); then final rmsnorm, vocab head and the global
 * argmax (lowest index wins ties) into *token.  head_dim must be 128 and
 * n_q_heads / n_kv_heads one of 1, 2, 4, 8, 16.  Every tensor-parallel degree computes
 * the single-GPU step bit for bit (hidden state and token): the row-parallel Wo / Wd sums
 * follow one canonical order -- the row cut into up to 8 column segments (the shards at
 * the largest degree), each summed in a fixed order, the segments in a pairwise tree,
 * the ranks added in the same tree, then the residual -- and every RMSNorm uses one fixed
 * sum-of-squares order.  With collective = 0 the all-reduces are fused into the Wo/Wd
 * GEMVs and the following RMSNorm over NVLink peer memory (up to 8 ranks); with
 * collective = 1 the same exchange words travel through ncclAllGather between the
 * kernels (same bits, the baseline).  All launches and NCCL collectives go on the
 * caller's stream (graph-capturable).
 * ------------------------------------------------------------------------- */
typedef struct qg_decoder_dims {
  uint32_t layers, hidden, n_q_heads, n_kv_heads, head_dim, ffn, vocab, ctx_max;
  float eps, rope_base;
  int attn_fmt, ffn_fmt, down_fmt, head_fmt;
  uint32_t tp_rank, tp_size;
  uint32_t collective;  /* tp_size > 1: 0 = exchanges fused into the GEMVs over NVLink peer
                           memory (CUDA IPC), 1 = the same words moved by ncclAllGather */
} qg_decoder_dims;

typedef struct qg_decoder_layer {
  const float* attn_norm;
  const float* ffn_norm;
  const uint8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
  const uint8_t *wq_meta, *wk_meta, *wv_meta, *wo_meta, *wg_meta, *wu_meta, *wd_meta;
  void* k_cache;
  void* v_cache;
} qg_decoder_layer;

typedef struct qg_decoder_s* qg_decoder;

/* NCCL unique id (128 bytes) for rank 0 to share with the other ranks. */
cudaError_t qg_nccl_unique_id(void* id_out);
cudaError_t qg_decoder_workspace_bytes(const qg_decoder_dims* d, size_t* bytes);
cudaError_t qg_decoder_shard(const qg_decoder_dims* d, uint32_t* q_rows, uint32_t* kv_rows,
                             uint32_t* ffn_rows, uint32_t* vocab_rows, uint32_t* vocab_offset);
/* Bytes of a rank's exchange region (0 for tp_size 1). */
cudaError_t qg_decoder_exchange_bytes(const qg_decoder_dims* d, size_t* bytes);
/* Collective over the tp_size ranks when tp_size > 1 (NCCL communicator setup).  The
 * exchange region is allocated with cudaMalloc and shared through CUDA IPC. */
cudaError_t qg_decoder_create(const qg_decoder_dims* d, const qg_decoder_layer* layers,
                              const float* final_norm, const uint8_t* head,
                              const uint8_t* head_meta, void* workspace, const void* nccl_id,
                              qg_decoder* out);
/* The same with a caller-owned exchange region (tp_size > 1): 256-B aligned,
 * qg_decoder_exchange_bytes long, inside device memory from cudaMalloc (for example an
 * arena of the reference's VramSuperallocator, runtime/core/allocator/vram_superallocator.h:36-44),
 * whose allocation the peers map through CUDA IPC at the region's offset.  The library
 * allocates no device memory itself (NCCL's communicator aside). */
cudaError_t qg_decoder_create_in(const qg_decoder_dims* d, const qg_decoder_layer* layers,
                                 const float* final_norm, const uint8_t* head,
                                 const uint8_t* head_meta, void* workspace, void* exchange,
                                 const void* nccl_id, qg_decoder* out);
/* One decode step at position `pos` (0 <= pos < ctx_max), baked into the launches. */
cudaError_t qg_decoder_step(qg_decoder dec, const float* x, uint32_t pos, uint32_t* token,
                            cudaStream_t stream);
/* One decode step whose position is read on the device: *pos_dev (RoPE angle and cache
 * slot), attention over [0, *pos_dev] with its grid sized for ctx_bucket positions
 * (1 <= ctx_bucket <= ctx_max); advance != 0 adds 1 to *pos_dev after the token is
 * chosen.  One graph captured per context bucket then serves every token whose position
 * is below the bucket (the "one captured graph per decode step and bucket" of the
 * reference's graph runner, runtime/core/graphs/cuda_graph_bucket.h:70-139).  A position
 * at or past the bucket writes nothing to the caches and sets QG_ERR_POSITION. */
cudaError_t qg_decoder_step_at(qg_decoder dec, const float* x, uint32_t* pos_dev,
                               uint32_t ctx_bucket, uint32_t advance, uint32_t* token,
                               cudaStream_t stream);
/* Device pointers of the last step's final hidden state and this rank's logits. */
cudaError_t qg_decoder_views(qg_decoder dec, float** hidden, float** logits);
/* Device pointers of the last step's vectors of its last layer (no reference
 * counterpart; for stage-by-stage checks and debugging): the layer's input (the residual
 * stream, full width), this rank's Q/K/V rows before RoPE, its attention output, the
 * residual after the attention block (full width), its gate / up / silu(gate)*up rows,
 * the final hidden state and this rank's logits.  The workspace is reused by the next
 * step.  cudaErrorNotReady before the first step. */
typedef struct qg_decoder_stage_views {
  float *layer_input, *q, *k, *v, *attn, *x1, *g, *u, *a, *hidden, *logits;
} qg_decoder_stage_views;
cudaError_t qg_decoder_stage_buffers(qg_decoder dec, qg_decoder_stage_views* views);
cudaError_t qg_decoder_destroy(qg_decoder dec);

/* ---------------------------------------------------------------------------
 * GGUF ingest (host code; the reference's reader is runtime/apps/gguf_probe/main.cpp:124-631):
 * header, metadata (general.alignment, general.architecture), tensor infos, the data
 * section offset, tensor spans and the probe's validation (supported ggml type, block-
 * aligned element count, span >= expected bytes with padding < alignment).  Tensor bytes
 * are read into host memory; qgemv_b200/manifest.py writes them as resident packs.
 * Errors: cudaErrorFileNotFound (open), cudaErrorInvalidValue (not GGUF, truncated,
 * bad argument), cudaErrorInvalidSymbol (qg_gguf_find: no such tensor).
 * ------------------------------------------------------------------------- */
typedef struct qg_gguf_s* qg_gguf;
typedef struct qg_gguf_info {
  uint32_t version;
  uint64_t tensor_count, metadata_count;
  uint64_t tensor_info_end_offset, tensor_data_offset, tensor_data_alignment;
  uint64_t supported_tensors, valid_tensors, expected_data_bytes;
  char architecture[64];
} qg_gguf_info;
typedef struct qg_gguf_tensor_info {
  char name[256];
  uint32_t ggml_type;        /* 12 Q4_K, 13 Q5_K, 21 IQ3_S, 22 IQ2_S, 0 F32, 1 F16, 8 Q8_0 */
  uint32_t n_dims;
  uint64_t dims[4];          /* GGUF order: dims[0] = columns */
  uint64_t offset;           /* relative to the data section */
  uint64_t absolute_offset;  /* in the file */
  uint64_t span_bytes;       /* to the next tensor (or the end of the file) */
  uint64_t data_bytes;       /* expected bytes of the type and dims (0: unsupported type) */
  uint32_t block_size, type_size;
  uint32_t valid;
} qg_gguf_tensor_info;
cudaError_t qg_gguf_open(const char* path, qg_gguf* out);
cudaError_t qg_gguf_summary(qg_gguf g, qg_gguf_info* info);
cudaError_t qg_gguf_tensor(qg_gguf g, uint64_t index, qg_gguf_tensor_info* out);
cudaError_t qg_gguf_find(qg_gguf g, const char* name, uint64_t* index);
/* `bytes` must equal the tensor's data_bytes; the tensor must be valid. */
cudaError_t qg_gguf_read(qg_gguf g, uint64_t index, void* dst, uint64_t bytes);
cudaError_t qg_gguf_close(qg_gguf g);

/* Reads the library's device error word (QG_ERR_* bits) for the current device and
 * clears it.  Synchronizes the device.  Returns the cudaError_t of the read. */
cudaError_t qg_get_error(uint32_t* error_bits);

/* Number of SMs and launch configuration the GEMV uses for a shape, for
 * measurement code: grid CTAs, threads per CTA, rows per tile and pipeline stages. */
cudaError_t qg_gemv_plan(int fmt, uint32_t rows, uint32_t cols, uint32_t* grid,
                         uint32_t* threads, uint32_t* rows_per_tile, uint32_t* stages);
/* The same plan for a device of `sms` SMs, computed on the host without a device
 * (capacity planning; sms 0 plans for one SM). */
cudaError_t qg_gemv_plan_sms(int fmt, uint32_t rows, uint32_t cols, uint32_t sms, uint32_t* grid,
                             uint32_t* threads, uint32_t* rows_per_tile, uint32_t* stages);

#ifdef __cplusplus
}
#endif

#endif /* QGEMV_B200_H_ */
