// qg_host.h -- host-side interfaces shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/qgemv_b200.h"

namespace qg {

// Every kernel of the library is launched with programmatic stream serialization:
// it may start while the previous kernel on the stream finishes, and waits
// (griddepcontrol.wait) before it reads that kernel's output.  Captured into a CUDA
// graph this becomes a programmatic dependency edge.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Tensor-parallel exchange of a GEMV's output over NVLink peer memory (qg_decode.cu):
// every output row is stored into each rank's exchange buffer (this rank's slot, epoch
// parity half) as one 64-bit word (epoch << 32 | value bits), so a reader knows a word
// is current from the word itself -- no fence, counter or flag.  The buffers are peer
// pointers obtained through CUDA IPC.
constexpr uint32_t kMaxExchangeRanks = 8;
struct GemvExchange {
  uint64_t* out[kMaxExchangeRanks];   // per destination rank: this rank's slot, parity 0
  const uint32_t* epoch;              // exchanges completed on this GPU (the gather advances it)
  uint32_t n;                         // ranks (0: no exchange)
  uint32_t stride;                    // words from parity 0 to parity 1
};

// Launch configuration of the tiled GEMV for one shape (see qg_gemv.cu).
struct GemvPlan {
  uint32_t grid, threads, group, rpp, passes, rows_per_tile, num_tiles, stages;
  uint32_t stage_bytes, meta_off, red_off, table_off, stage_off, smem_bytes;
  uint32_t stage_passes, stage_rows, tiled;
};

// Tiled (TMA-pipelined) plan; .tiled == 0 when the shape cannot be staged that way.
// Row sums reduce lane groups of gcd(cols / 64, group_cap) chunks.
GemvPlan plan_gemv(int fmt, uint32_t rows, uint32_t cols, int sms, uint32_t group_cap = 32u);
// Plan of the all-thread-copy kernel used for packs that are not 16-B aligned.
GemvPlan plan_staged(int fmt, uint32_t rows, uint32_t cols, int sms);

// y = W x (+ residual); optional reference KV page write with the token read on
// the device before the launch's first row is stored.
// `act` (optional) is x prepared by launch_act_prepare; the kernel then skips its own
// quantization of x.
cudaError_t launch_gemv(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                        const void* act, float* y, const float* residual, float* kv,
                        const uint32_t* token, uint64_t kv_words, uint32_t page_words,
                        uint32_t active_pages, uint32_t rows, uint32_t cols, cudaStream_t stream);

// Up to 3 matrices of one format and width reading the same x, in one launch.
cudaError_t launch_gemv_multi(int fmt, uint32_t nseg, const uint8_t* const* payload,
                              const uint8_t* const* meta, float* const* y, const uint32_t* rows,
                              uint32_t cols, const float* x, const void* act, cudaStream_t stream);

// Multi-vector GEMV on the CUDA cores (qg_gemv_batch.cu): Y[v] = W X[v] for v < nvec
// (1..8), X[v] at x + v * x_stride, Y[v] at y + v * y_stride; one launch per column
// slice, chained on the stream.  Plan of one launch (every slice of a matrix shares it).
struct BatchPlan {
  uint32_t slices, warps, q, units, stages, slot_p, slot_m, stage_bytes;
  uint32_t table_off, red_off, xs_off, stage_off, smem, ok;
};
BatchPlan plan_gemv_batch(int fmt, uint32_t nvec, uint32_t rows, uint32_t cols);
// Shapes and alignments the multi-vector kernel takes (16-B aligned payload / metadata).
bool gemv_batch_ok(int fmt, const uint8_t* payload, const uint8_t* meta, uint32_t rows, uint32_t cols);
cudaError_t launch_gemv_batch(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                              float* y, uint32_t nvec, uint32_t x_stride, uint32_t y_stride,
                              uint32_t rows, uint32_t cols, cudaStream_t stream);
// First batch size qg_gemm_batched runs on the tensor cores (QG_TC_MIN_BATCH overrides).
uint32_t tc_min_batch();
// Y = W X for `batch` vectors (X [batch][cols], Y [batch][rows]) on the CUDA cores:
// one weight pass per group of up to 8 vectors.
cudaError_t launch_gemv_vectors(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                                float* y, uint32_t batch, uint32_t rows, uint32_t cols,
                                cudaStream_t stream);

// Batched-slice helpers (row r of every [rows][n] operand): h[r] = rmsnorm(x[r]) * w
// (norm_prepare's sum-of-squares order), a = silu(gate) * up, out = x + y.
cudaError_t launch_norm_rows(const float* x, const float* w, uint32_t n, float eps, float* h,
                             uint32_t rows, cudaStream_t stream);
cudaError_t launch_silu_gate_rows(const float* gate, const float* up, size_t total, float* a,
                                  cudaStream_t stream);
cudaError_t launch_add_rows(const float* x, const float* y, size_t total, float* out,
                            cudaStream_t stream);
// Y = W X for `batch` vectors with qg_gemm_batched's routing (batch-1 GEMV, CUDA-core
// multi-vector GEMV below the tensor-core threshold, tensor-core tiles above for the
// four GGUF formats); batched_gemm_ws_bytes is the tensor-core workspace it needs.
size_t batched_gemm_ws_bytes(int fmt, uint32_t batch, uint32_t rows, uint32_t cols);
cudaError_t launch_batched_gemm(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                                float* y, uint32_t batch, uint32_t rows, uint32_t cols,
                                void* workspace, cudaStream_t stream);

// Bytes of a prepared activation of `cols` values (176 per 64 columns).
inline size_t act_bytes(uint32_t cols) { return static_cast<size_t>(cols / 64u) * 176u; }
cudaError_t launch_act_prepare(const float* x, uint32_t cols, void* act, cudaStream_t stream);

// token = (argmax(v[0:n]) + offset + add_token * token) % modulus (one CTA).
cudaError_t launch_argmax_token(const float* v, uint32_t n, uint32_t* token, uint32_t offset,
                                uint32_t add_token, uint32_t modulus, cudaStream_t stream);

// The reference's feedback kernels (modes in qg_aux.cu).
cudaError_t launch_feedback(uint32_t mode, const float* logits, float* act, float* cache,
                            const float* gate, uint32_t rows, uint32_t cols, uint32_t cache_cols,
                            float eps, uint32_t accumulate, cudaStream_t stream);

cudaError_t launch_dequant(int fmt, const uint8_t* payload, const uint8_t* meta,
                           uint64_t first_block, uint64_t count, float* out, cudaStream_t stream);

cudaError_t launch_weighted_rmsnorm(const float* x, const float* w, uint32_t n, float eps,
                                    float* y, cudaStream_t stream);

cudaError_t launch_silu_gate(const float* gate, const float* up, uint32_t n, float* h,
                             cudaStream_t stream);

// Canonical summation order of a row-parallel matrix's rows: the full row (all ranks'
// columns) is 8 (or fewer, a power of two) segments, one tensor-parallel shard at the
// largest degree each; a rank's launch covers `nseg` consecutive segments of
// `seg_chunks` 64-column chunks.  Each segment is summed in a fixed order, the segments
// in a pairwise tree, and the exchange gather adds the ranks in the same tree, so every
// tensor-parallel degree produces the single-GPU row sums bit for bit.
struct GemvCanon {
  uint32_t seg_chunks;
  uint32_t nseg;
};

// y = W x (+ residual) with canonical row sums (tiled kernel only; returns
// cudaErrorNotSupported for shapes or alignments that need the fallback kernels).
cudaError_t launch_gemv_canonical(int fmt, const uint8_t* payload, const uint8_t* meta,
                                  const float* x, const void* act, float* y, const float* residual,
                                  uint32_t rows, uint32_t cols, const GemvCanon& canon,
                                  cudaStream_t stream);
// The same, whose rows are also exchanged to every rank.
cudaError_t launch_gemv_exchange(int fmt, const uint8_t* payload, const uint8_t* meta,
                                 const float* x, const void* act, float* y, const float* residual,
                                 uint32_t rows, uint32_t cols, const GemvExchange& ex,
                                 const GemvCanon& canon, cudaStream_t stream);
// Reads every rank's slot, waiting (bounded) for each word of epoch+1, adds the ranks in
// a pairwise tree and then to `residual` (optional) into x_out, advances the epoch, then
// RMSNorm*w and h's int8 planes like launch_norm_prepare.
cudaError_t launch_gather_norm_prepare(const uint64_t* buf, uint32_t* epoch, uint32_t nsrc,
                                       uint32_t stride, const float* residual, const float* w,
                                       uint32_t n, float eps, float* x_out, float* h, void* act,
                                       cudaStream_t stream);
cudaError_t launch_norm_prepare(const float* x, const float* w, uint32_t n, float eps, float* h,
                                void* act, cudaStream_t stream);
// a = silu(gate) * up (+ a's prepared activation).
cudaError_t launch_silu_gate_prepare(const float* gate, const float* up, uint32_t n, float* a,
                                     void* act, cudaStream_t stream);

int device_sm_count();

}  // namespace qg
