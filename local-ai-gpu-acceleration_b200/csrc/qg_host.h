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

// Launch configuration of the tiled GEMV for one shape (see qg_gemv.cu).
struct GemvPlan {
  uint32_t grid, threads, group, rpp, passes, rows_per_tile, num_tiles, stages;
  uint32_t stage_bytes, meta_off, red_off, table_off, stage_off, smem_bytes;
  uint32_t stage_passes, stage_rows, tiled;
};

// Tiled (TMA-pipelined) plan; .tiled == 0 when the shape cannot be staged that way.
GemvPlan plan_gemv(int fmt, uint32_t rows, uint32_t cols, int sms);
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

// h = x * inv_rms(x) * w (+ h's prepared activation); one CTA.
cudaError_t launch_norm_prepare(const float* x, const float* w, uint32_t n, float eps, float* h,
                                void* act, cudaStream_t stream);
// a = silu(gate) * up (+ a's prepared activation).
cudaError_t launch_silu_gate_prepare(const float* gate, const float* up, uint32_t n, float* a,
                                     void* act, cudaStream_t stream);

int device_sm_count();

}  // namespace qg
