// qg_abi.cu -- the extern "C" boundary of libqgemv_b200.so (include/qgemv_b200.h).
//
// The rtxllm_launch_* functions keep the reference launchers' contract
// (runtime/kernels/decode/decode_kernels.cu:3106-3243, 3956-4639): same argument
// validation and return codes, logits for the launched rows, the KV page write with
// the pre-update token, then the argmax token update -- so the reference's apps
// link against this library unchanged.  They differ only in how the work is done:
// every Q4_K "variant" launcher runs the same tiled sm_100a kernel, because the
// variants were alternative implementations of one function.
#include "qg_host.h"

namespace qg {
extern __device__ unsigned int g_error_word;
}

namespace {

constexpr uint32_t kTokenModulus = 32000u;  // argmax_token_kernel, decode_kernels.cu:3029

bool valid_fmt(int fmt) { return fmt >= 0 && fmt < QG_FMT_COUNT; }

// Matvec + KV write + token update, as every reference decode launcher does.
cudaError_t decode_stage(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                         float* y, float* kv, uint32_t* token, uint32_t rows, uint32_t cols,
                         uint32_t kv_words, uint32_t page_words, uint32_t active_pages,
                         cudaStream_t stream) {
  cudaError_t e = qg::launch_gemv(fmt, payload, meta, x, nullptr, y, nullptr, kv, token, kv_words,
                                  page_words, active_pages, rows, cols, stream);
  if (e != cudaSuccess) return e;
  if (token == nullptr) return cudaSuccess;
  return qg::launch_argmax_token(y, rows, token, 1u, 1u, kTokenModulus, stream);
}

// Q4_K launchers of the reference do not validate; a zero-row grid is the
// reference's launch error, and columns beyond the last whole block are ignored.
cudaError_t q4k_compat(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                       float* y, float* kv, uint32_t* token, uint32_t rows, uint32_t cols,
                       uint32_t kv_words, uint32_t page_words, uint32_t active_pages,
                       cudaStream_t stream) {
  if (rows == 0u) return cudaErrorInvalidConfiguration;
  return decode_stage(fmt, payload, meta, x, y, kv, token, rows, cols & ~255u, kv_words,
                      page_words, active_pages, stream);
}

// IQ/Q5_K probe launchers: validate like decode_kernels.cu:4046-4048 and launch
// min(rows, rows_limit) rows.
cudaError_t probe_compat(int fmt, const uint8_t* blocks, const float* x, float* y, float* kv,
                         uint32_t* token, uint32_t rows, uint32_t cols, uint32_t rows_limit,
                         uint32_t kv_words, uint32_t page_words, uint32_t active_pages,
                         cudaStream_t stream) {
  if (rows == 0u || cols == 0u || rows_limit == 0u || (cols % 256u) != 0u) {
    return cudaErrorInvalidValue;
  }
  const uint32_t launched = rows_limit < rows ? rows_limit : rows;
  return decode_stage(fmt, blocks, nullptr, x, y, kv, token, launched, cols, kv_words,
                      page_words, active_pages, stream);
}

}  // namespace

extern "C" {

#define QG_Q4K_RAW_LAUNCHER(NAME)                                                         \
  cudaError_t NAME(const uint8_t* q4k_blocks, const float* activation, float* logits,     \
                   float* kv, uint32_t* token, uint32_t rows, uint32_t cols,              \
                   uint32_t kv_words, uint32_t page_words, uint32_t active_pages,         \
                   cudaStream_t stream) {                                                 \
    return q4k_compat(QG_FMT_Q4K_RAW, q4k_blocks, nullptr, activation, logits, kv, token, \
                      rows, cols, kv_words, page_words, active_pages, stream);            \
  }
QG_Q4K_RAW_LAUNCHER(rtxllm_launch_q4k_matvec_decode)
QG_Q4K_RAW_LAUNCHER(rtxllm_launch_q4k_matvec_decode_shared)
QG_Q4K_RAW_LAUNCHER(rtxllm_launch_q4k_matvec_decode_warp)
QG_Q4K_RAW_LAUNCHER(rtxllm_launch_q4k_matvec_decode_warp_broadcast)
QG_Q4K_RAW_LAUNCHER(rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4)
QG_Q4K_RAW_LAUNCHER(rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x2)
QG_Q4K_RAW_LAUNCHER(rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x4)
#undef QG_Q4K_RAW_LAUNCHER

cudaError_t rtxllm_launch_q4k_matvec_decode_predecoded_vec4x4(
    const uint8_t* q4k_blocks, const float* /*q4k_scale_min_pairs*/, const float* activation,
    float* logits, float* kv, uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words,
    uint32_t page_words, uint32_t active_pages, cudaStream_t stream) {
  return q4k_compat(QG_FMT_Q4K_RAW, q4k_blocks, nullptr, activation, logits, kv, token, rows, cols,
                    kv_words, page_words, active_pages, stream);
}

cudaError_t rtxllm_launch_q4k_matvec_decode_split_predecoded_vec4x4(
    const uint8_t* q4k_payload, const float* q4k_scale_min_pairs, const float* activation,
    float* logits, float* kv, uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words,
    uint32_t page_words, uint32_t active_pages, cudaStream_t stream) {
  return q4k_compat(QG_FMT_Q4K_SPLIT_PREDECODED, q4k_payload,
                    reinterpret_cast<const uint8_t*>(q4k_scale_min_pairs), activation, logits, kv,
                    token, rows, cols, kv_words, page_words, active_pages, stream);
}

cudaError_t rtxllm_launch_q4k_matvec_decode_split_half_vec4x4(
    const uint8_t* q4k_payload, const uint16_t* q4k_scale_min_half_pairs, const float* activation,
    float* logits, float* kv, uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words,
    uint32_t page_words, uint32_t active_pages, cudaStream_t stream) {
  return q4k_compat(QG_FMT_Q4K_SPLIT_HALF, q4k_payload,
                    reinterpret_cast<const uint8_t*>(q4k_scale_min_half_pairs), activation, logits,
                    kv, token, rows, cols, kv_words, page_words, active_pages, stream);
}

cudaError_t rtxllm_launch_q4k_matvec_decode_split_compact_vec4x4(
    const uint8_t* q4k_payload, const uint8_t* q4k_compact_meta, const float* activation,
    float* logits, float* kv, uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words,
    uint32_t page_words, uint32_t active_pages, cudaStream_t stream) {
  return q4k_compat(QG_FMT_Q4K_SPLIT_COMPACT, q4k_payload, q4k_compact_meta, activation, logits,
                    kv, token, rows, cols, kv_words, page_words, active_pages, stream);
}

cudaError_t rtxllm_launch_q4k_matvec_decode_split_native_vec4x4(
    const uint8_t* q4k_payload, const uint8_t* q4k_native_meta, const float* activation,
    float* logits, float* kv, uint32_t* token, uint32_t rows, uint32_t cols, uint32_t kv_words,
    uint32_t page_words, uint32_t active_pages, cudaStream_t stream) {
  return q4k_compat(QG_FMT_Q4K_SPLIT_NATIVE, q4k_payload, q4k_native_meta, activation, logits, kv,
                    token, rows, cols, kv_words, page_words, active_pages, stream);
}

cudaError_t rtxllm_launch_q5k_matvec_decode_probe(
    const uint8_t* q5k_blocks, const float* activation, float* logits, float* kv, uint32_t* token,
    uint32_t rows, uint32_t cols, uint32_t rows_limit, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream) {
  return probe_compat(QG_FMT_Q5K, q5k_blocks, activation, logits, kv, token, rows, cols, rows_limit,
                      kv_words, page_words, active_pages, stream);
}

cudaError_t rtxllm_launch_iq2s_matvec_probe(const uint8_t* iq2s_blocks, const float* activation,
                                            float* logits, uint32_t rows, uint32_t cols,
                                            uint32_t rows_limit, cudaStream_t stream) {
  return probe_compat(QG_FMT_IQ2S, iq2s_blocks, activation, logits, nullptr, nullptr, rows, cols,
                      rows_limit, 0u, 0u, 0u, stream);
}

cudaError_t rtxllm_launch_iq2s_matvec_decode_probe(
    const uint8_t* iq2s_blocks, const float* activation, float* logits, float* kv, uint32_t* token,
    uint32_t rows, uint32_t cols, uint32_t rows_limit, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream) {
  return probe_compat(QG_FMT_IQ2S, iq2s_blocks, activation, logits, kv, token, rows, cols,
                      rows_limit, kv_words, page_words, active_pages, stream);
}

cudaError_t rtxllm_launch_iq3s_matvec_decode_probe(
    const uint8_t* iq3s_blocks, const float* activation, float* logits, float* kv, uint32_t* token,
    uint32_t rows, uint32_t cols, uint32_t rows_limit, uint32_t kv_words, uint32_t page_words,
    uint32_t active_pages, cudaStream_t stream) {
  return probe_compat(QG_FMT_IQ3S, iq3s_blocks, activation, logits, kv, token, rows, cols,
                      rows_limit, kv_words, page_words, active_pages, stream);
}

cudaError_t rtxllm_launch_output_token_sample(const float* logits, uint32_t* token, uint32_t rows,
                                              uint32_t vocab_size, uint32_t token_offset,
                                              cudaStream_t stream) {
  if (logits == nullptr || token == nullptr || rows == 0u || vocab_size == 0u) {
    return cudaErrorInvalidValue;
  }
  return qg::launch_argmax_token(logits, rows, token, token_offset, 0u, vocab_size, stream);
}

cudaError_t rtxllm_launch_rmsnorm_feedback(const float* logits, float* activation, uint32_t rows,
                                           uint32_t cols, float epsilon, cudaStream_t stream) {
  return qg::launch_feedback(0u, logits, activation, nullptr, nullptr, rows, cols, 0u, epsilon, 0u,
                             stream);
}

cudaError_t rtxllm_launch_silu_rmsnorm_feedback(const float* logits, float* activation,
                                                uint32_t rows, uint32_t cols, float epsilon,
                                                cudaStream_t stream) {
  return qg::launch_feedback(1u, logits, activation, nullptr, nullptr, rows, cols, 0u, epsilon, 0u,
                             stream);
}

cudaError_t rtxllm_launch_rmsnorm_feedback_with_silu_cache(const float* logits, float* activation,
                                                           float* silu_cache, uint32_t rows,
                                                           uint32_t cols, float epsilon,
                                                           cudaStream_t stream) {
  return qg::launch_feedback(2u, logits, activation, silu_cache, nullptr, rows, cols, 0u, epsilon,
                             0u, stream);
}

cudaError_t rtxllm_launch_gated_silu_rmsnorm_feedback(const float* logits, const float* silu_cache,
                                                      float* activation, uint32_t rows,
                                                      uint32_t cache_cols, uint32_t cols,
                                                      float epsilon, cudaStream_t stream) {
  if (cache_cols == 0u) return cudaSuccess;  // the reference kernel writes nothing
  return qg::launch_feedback(3u, logits, activation, const_cast<float*>(silu_cache), nullptr, rows,
                             cols, cache_cols, epsilon, 0u, stream);
}

cudaError_t rtxllm_launch_rmsnorm_silu_cache(const float* logits, float* silu_cache, uint32_t rows,
                                             uint32_t cache_cols, float epsilon,
                                             uint32_t accumulate, cudaStream_t stream) {
  if (cache_cols == 0u) return cudaErrorInvalidValue;
  return qg::launch_feedback(5u, logits, nullptr, silu_cache, nullptr, rows, cache_cols,
                             cache_cols, epsilon, accumulate, stream);
}

cudaError_t rtxllm_launch_rmsnorm_cache(const float* logits, float* cache, uint32_t rows,
                                        uint32_t cache_cols, float epsilon, uint32_t accumulate,
                                        cudaStream_t stream) {
  if (cache_cols == 0u) return cudaErrorInvalidValue;
  return qg::launch_feedback(4u, logits, nullptr, cache, nullptr, rows, cache_cols, cache_cols,
                             epsilon, accumulate, stream);
}

cudaError_t rtxllm_launch_rmsnorm_cache_and_gated_product(
    const float* logits, const float* gate_cache, float* up_cache, float* activation,
    uint32_t rows, uint32_t cache_cols, uint32_t output_cols, float epsilon, uint32_t accumulate,
    cudaStream_t stream) {
  if (cache_cols == 0u || output_cols == 0u) return cudaErrorInvalidValue;
  return qg::launch_feedback(6u, logits, activation, up_cache, gate_cache, rows, output_cols,
                             cache_cols, epsilon, accumulate, stream);
}

// ---------------------------------------------------------------------------
// New entry points.

static bool gemv_args_ok(int fmt, const uint8_t* payload, const uint8_t* meta, const void* x,
                         const void* y, uint32_t rows, uint32_t cols) {
  if (!valid_fmt(fmt) || payload == nullptr || x == nullptr || y == nullptr) return false;
  if (qg_meta_bytes_per_block(fmt) != 0u && meta == nullptr) return false;
  return rows != 0u && cols != 0u && (cols % 256u) == 0u;
}

cudaError_t qg_gemv(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x, float* y,
                    uint32_t rows, uint32_t cols, cudaStream_t stream) {
  if (!gemv_args_ok(fmt, payload, meta, x, y, rows, cols)) return cudaErrorInvalidValue;
  return qg::launch_gemv(fmt, payload, meta, x, nullptr, y, nullptr, nullptr, nullptr, 0u, 0u, 0u,
                         rows, cols, stream);
}

cudaError_t qg_decode_stage(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                            float* y, float* kv, uint32_t* token, uint32_t rows, uint32_t cols,
                            uint32_t kv_words, uint32_t page_words, uint32_t active_pages,
                            cudaStream_t stream) {
  if (!gemv_args_ok(fmt, payload, meta, x, y, rows, cols) || token == nullptr) {
    return cudaErrorInvalidValue;
  }
  return decode_stage(fmt, payload, meta, x, y, kv, token, rows, cols, kv_words, page_words,
                      active_pages, stream);
}

cudaError_t qg_gemv_batched(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                            float* y, uint32_t batch, uint32_t rows, uint32_t cols,
                            cudaStream_t stream) {
  if (!gemv_args_ok(fmt, payload, meta, x, y, rows, cols) || batch == 0u || batch > 32u) {
    return cudaErrorInvalidValue;
  }
  return qg::launch_gemv_vectors(fmt, payload, meta, x, y, batch, rows, cols, stream);
}

cudaError_t qg_act_bytes(uint32_t cols, size_t* bytes) {
  if (bytes == nullptr || cols == 0u || (cols % 256u) != 0u) return cudaErrorInvalidValue;
  *bytes = qg::act_bytes(cols);
  return cudaSuccess;
}

cudaError_t qg_act_prepare(const float* x, uint32_t cols, void* act, cudaStream_t stream) {
  if (x == nullptr || act == nullptr || cols == 0u || (cols % 256u) != 0u ||
      (reinterpret_cast<uintptr_t>(act) & 15u) != 0u ||
      (reinterpret_cast<uintptr_t>(x) & 7u) != 0u) {
    return cudaErrorInvalidValue;
  }
  return qg::launch_act_prepare(x, cols, act, stream);
}

cudaError_t qg_gemv_act(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                        const void* act, float* y, uint32_t rows, uint32_t cols,
                        cudaStream_t stream) {
  if (!gemv_args_ok(fmt, payload, meta, x, y, rows, cols) ||
      (act != nullptr && (reinterpret_cast<uintptr_t>(act) & 15u) != 0u)) {
    return cudaErrorInvalidValue;
  }
  return qg::launch_gemv(fmt, payload, meta, x, act, y, nullptr, nullptr, nullptr, 0u, 0u, 0u,
                         rows, cols, stream);
}

cudaError_t qg_dequantize(int fmt, const uint8_t* payload, const uint8_t* meta,
                          uint64_t first_block, uint64_t block_count, float* out,
                          cudaStream_t stream) {
  if (!valid_fmt(fmt) || payload == nullptr || out == nullptr || block_count == 0u ||
      (qg_meta_bytes_per_block(fmt) != 0u && meta == nullptr)) {
    return cudaErrorInvalidValue;
  }
  return qg::launch_dequant(fmt, payload, meta, first_block, block_count, out, stream);
}

cudaError_t qg_argmax_token(const float* values, uint32_t n, uint32_t* token,
                            uint32_t token_offset, uint32_t add_token, uint32_t modulus,
                            cudaStream_t stream) {
  if (values == nullptr || token == nullptr || n == 0u || modulus == 0u) {
    return cudaErrorInvalidValue;
  }
  return qg::launch_argmax_token(values, n, token, token_offset, add_token, modulus, stream);
}

cudaError_t qg_get_error(uint32_t* error_bits) {
  if (error_bits == nullptr) return cudaErrorInvalidValue;
  unsigned int v = 0u;
  cudaError_t e = cudaMemcpyFromSymbol(&v, qg::g_error_word, sizeof(v));
  if (e != cudaSuccess) return e;
  const unsigned int zero = 0u;
  e = cudaMemcpyToSymbol(qg::g_error_word, &zero, sizeof(zero));
  *error_bits = v;
  return e;
}

cudaError_t qg_gemv_plan(int fmt, uint32_t rows, uint32_t cols, uint32_t* grid, uint32_t* threads,
                         uint32_t* rows_per_tile, uint32_t* stages) {
  return qg_gemv_plan_sms(fmt, rows, cols, static_cast<uint32_t>(qg::device_sm_count()), grid,
                          threads, rows_per_tile, stages);
}

cudaError_t qg_gemv_plan_sms(int fmt, uint32_t rows, uint32_t cols, uint32_t sms, uint32_t* grid,
                             uint32_t* threads, uint32_t* rows_per_tile, uint32_t* stages) {
  if (!valid_fmt(fmt) || rows == 0u || cols < 256u || (cols % 256u) != 0u) {
    return cudaErrorInvalidValue;
  }
  const qg::GemvPlan p = qg::plan_gemv(fmt, rows, cols, static_cast<int>(sms));
  if (grid) *grid = p.grid;
  if (threads) *threads = p.threads;
  if (rows_per_tile) *rows_per_tile = p.rows_per_tile;
  if (stages) *stages = p.stages;
  return cudaSuccess;
}

}  // extern "C"
