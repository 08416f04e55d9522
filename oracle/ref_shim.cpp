// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's own CPU reference functions, unmodified, into
// oracle/_ref/libref_oracle.so and gives them C linkage.  The reference keeps
// them in an anonymous namespace inside
// runtime/apps/mixed_sequence_benchmark_runner/main.cpp:1075-1500, so this
// translation unit includes that file (read-only, from the reference tree; its
// main() is renamed) and wraps the functions below.  Nothing here is shipped:
// the wrappers are called by tests/golden/make_golden.py (golden vectors),
// tests/test_oracle_cpu.py (pinning oracle/qoracle.c) and bench.py's CPU
// baseline leg.  Built by oracle/Makefile; needs the reference tree at build
// time only.
#define main reference_mixed_main
#include "runtime/apps/mixed_sequence_benchmark_runner/main.cpp"
#undef main

#include <chrono>
#include <thread>

namespace {

// Pack formats, numbered as include/qgemv_b200.h's qg_format.
const char* q4k_kernel_name(int fmt) {
  switch (fmt) {
    case 1: return "split-predecoded";
    case 2: return "split-half";
    case 3: return "split-compact";
    case 0:  // raw 144-B blocks are split-native with meta = block[0:16]
    case 4: return "split-native";
    default: return nullptr;
  }
}

Stage make_stage(int fmt, std::uint32_t rows, std::uint32_t cols) {
  Stage stage;
  stage.rows = rows;
  stage.cols = cols;
  if (fmt >= 0 && fmt <= 4) {
    stage.kind = StageKind::Q4K;
    stage.q4k.runtime_kernel = q4k_kernel_name(fmt);
    stage.type = "Q4_K";
  } else if (fmt == 5) {
    stage.kind = StageKind::Q5K;
    stage.type = "Q5_K";
  } else if (fmt == 6) {
    stage.kind = StageKind::IQ2S;
    stage.type = "IQ2_S";
  } else {
    stage.kind = StageKind::IQ3S;
    stage.type = "IQ3_S";
  }
  return stage;
}

std::uint32_t payload_block_bytes(int fmt) {
  switch (fmt) {
    case 0: return 144u;
    case 1: case 2: case 3: case 4: return 128u;
    case 5: return 176u;
    case 6: return 82u;
    case 7: return 110u;
    default: return 0u;
  }
}

std::uint32_t meta_block_bytes(int fmt) {
  switch (fmt) {
    case 1: return 64u;
    case 2: return 32u;
    case 3: return 20u;
    case 4: return 16u;
    default: return 0u;
  }
}

// The reference's Q4_K path reads split packs only; a raw 144-B block stream is
// handed to it as (payload = block[16:144], meta = block[0:16]), the byte-exact
// split-native form (tools/bench/q4k_resident_pack.py:104-106,141-145).
void split_raw_q4k(const std::uint8_t* blocks, std::uint64_t nblocks,
                   std::vector<std::uint8_t>& payload, std::vector<std::uint8_t>& meta) {
  payload.resize(nblocks * 128u);
  meta.resize(nblocks * 16u);
  for (std::uint64_t b = 0; b < nblocks; ++b) {
    std::memcpy(meta.data() + b * 16u, blocks + b * 144u, 16u);
    std::memcpy(payload.data() + b * 128u, blocks + b * 144u + 16u, 128u);
  }
}

void gather_rows(int fmt, const std::uint8_t* payload, const std::uint8_t* meta,
                 std::uint32_t cols, std::uint32_t row_begin, std::uint32_t row_end,
                 std::vector<std::uint8_t>& p, std::vector<std::uint8_t>& m) {
  const std::uint64_t bpr = cols / 256u;
  const std::uint64_t b0 = row_begin * bpr;
  const std::uint64_t nb = (row_end - row_begin) * bpr;
  if (fmt == 0) {
    split_raw_q4k(payload + b0 * 144u, nb, p, m);
    return;
  }
  const auto pb = payload_block_bytes(fmt);
  p.assign(payload + b0 * pb, payload + (b0 + nb) * pb);
  const auto mb = meta_block_bytes(fmt);
  if (mb != 0u) {
    m.assign(meta + b0 * mb, meta + (b0 + nb) * mb);
  } else {
    m.clear();
  }
}

}  // namespace

extern "C" {

// reference_stage_logits (main.cpp:1261-1309) over rows [row_begin, row_end).
int ref_stage_logits(int fmt, const std::uint8_t* payload, const std::uint8_t* meta,
                     const float* activation, std::uint32_t cols, std::uint32_t row_begin,
                     std::uint32_t row_end, float* out) {
  if (fmt < 0 || fmt > 7 || cols == 0u || cols % 256u != 0u || row_end < row_begin) {
    return 1;
  }
  std::vector<std::uint8_t> p, m;
  gather_rows(fmt, payload, meta, cols, row_begin, row_end, p, m);
  const Stage stage = make_stage(fmt, row_end - row_begin, cols);
  const std::vector<float> act(activation, activation + cols);
  const auto logits = reference_stage_logits(stage, p, m, act);
  std::memcpy(out, logits.data(), logits.size() * sizeof(float));
  return 0;
}

// Per-value dequantization: q4k_dequant_value / iq2s_dequant_value /
// iq3s_dequant_value / q5k_dequant_value (main.cpp:1133-1259).
int ref_dequant_blocks(int fmt, const std::uint8_t* payload, const std::uint8_t* meta,
                       std::uint64_t first_block, std::uint64_t block_count, float* out) {
  for (std::uint64_t b = 0; b < block_count; ++b) {
    const std::uint64_t bi = first_block + b;
    for (std::uint32_t v = 0; v < 256u; ++v) {
      float value = 0.0f;
      switch (fmt) {
        case 0:
          value = q4k_dequant_value(payload + bi * 144u + 16u, payload + bi * 144u,
                                    "split-native", v);
          break;
        case 1: case 2: case 3: case 4:
          value = q4k_dequant_value(payload + bi * 128u, meta + bi * meta_block_bytes(fmt),
                                    q4k_kernel_name(fmt), v);
          break;
        case 5: value = q5k_dequant_value(payload + bi * 176u, v); break;
        case 6: value = iq2s_dequant_value(payload + bi * 82u, v); break;
        case 7: value = iq3s_dequant_value(payload + bi * 110u, v); break;
        default: return 1;
      }
      out[b * 256u + v] = value;
    }
  }
  return 0;
}

// argmax_token (main.cpp:1311-1322).
std::uint32_t ref_argmax(const float* logits, std::uint32_t n) {
  return argmax_token(std::vector<float>(logits, logits + n));
}

// apply_reference_kv (main.cpp:1324-1341).
void ref_apply_kv(const float* logits, std::uint32_t rows, float* kv, std::uint64_t kv_words,
                  std::uint32_t token, std::uint32_t page_words, std::uint32_t active_pages) {
  std::vector<float> kvv(kv, kv + kv_words);
  apply_reference_kv(std::vector<float>(logits, logits + rows), kvv, token, page_words,
                     active_pages);
  std::memcpy(kv, kvv.data(), kv_words * sizeof(float));
}

// Feedback math (main.cpp:1363-1488).  kind: 0 rmsnorm, 1 silu_rmsnorm,
// 2 rmsnorm_with_silu_cache (writes act and cache), 3 gated_silu (reads cache),
// 4 rmsnorm_cache, 5 rmsnorm_silu_cache.  `accumulate` for kinds 4/5.
void ref_feedback(int kind, const float* logits, std::uint32_t rows, float* act,
                  std::uint32_t cols, float* cache, std::uint32_t cache_cols, float eps,
                  int accumulate) {
  const std::vector<float> lg(logits, logits + rows);
  std::vector<float> a(act, act + cols);
  std::vector<float> c(cache, cache + cache_cols);
  switch (kind) {
    case 0: apply_reference_rmsnorm_feedback(lg, a, cols, eps); break;
    case 1: apply_reference_silu_rmsnorm_feedback(lg, a, cols, eps); break;
    case 2: apply_reference_rmsnorm_feedback_with_silu_cache(lg, a, c, cols, eps); break;
    case 3: apply_reference_gated_silu_rmsnorm_feedback(lg, c, a, cols, eps); break;
    case 4: apply_reference_rmsnorm_cache(lg, c, cache_cols, eps, false, accumulate != 0); break;
    case 5: apply_reference_rmsnorm_cache(lg, c, cache_cols, eps, true, accumulate != 0); break;
    default: return;
  }
  std::memcpy(act, a.data(), cols * sizeof(float));
  if (cache_cols != 0u) {
    std::memcpy(cache, c.data(), std::min<std::size_t>(c.size(), cache_cols) * sizeof(float));
  }
}

// The CPU twin of rmsnorm_cache_and_gated_product (decode_kernels.cu:263-289) as the
// mixed runner's CPU reference applies it (main.cpp:2620-2633): the up cache gets the
// normalised logits (accumulated or not), then activation = gate cache x up cache
// (main.cpp:1459-1503).
void ref_cache_gated_product(const float* logits, std::uint32_t rows, const float* gate,
                             std::uint32_t gate_cols, float* up, std::uint32_t up_cols,
                             float* act, std::uint32_t cols, float eps, int accumulate) {
  const std::vector<float> lg(logits, logits + rows);
  const std::vector<float> g(gate, gate + gate_cols);
  std::vector<float> u(up, up + up_cols);
  std::vector<float> a(act, act + cols);
  apply_reference_rmsnorm_cache(lg, u, cols, eps, false, accumulate != 0);
  apply_reference_gated_cache_product(g, u, a, cols);
  std::memcpy(up, u.data(), std::min<std::size_t>(u.size(), up_cols) * sizeof(float));
  std::memcpy(act, a.data(), cols * sizeof(float));
}

// CPU baseline: time reference_stage_logits over rows [0, rows) split into
// `threads` contiguous row slices, one std::thread each (the reference function
// itself is single-threaded).  Payload slices are gathered before the clock
// starts.  Returns elapsed seconds, or -1 on bad arguments.
double ref_time_stage_logits(int fmt, const std::uint8_t* payload, const std::uint8_t* meta,
                             const float* activation, std::uint32_t rows, std::uint32_t cols,
                             std::uint32_t threads, float* out) {
  if (fmt < 0 || fmt > 7 || rows == 0u || cols == 0u || cols % 256u != 0u) return -1.0;
  if (threads == 0u) threads = 1u;
  if (threads > rows) threads = rows;
  std::vector<std::vector<std::uint8_t>> ps(threads), ms(threads);
  std::vector<Stage> stages;
  std::vector<std::uint32_t> begins(threads + 1u);
  for (std::uint32_t t = 0; t <= threads; ++t) {
    begins[t] = static_cast<std::uint32_t>((static_cast<std::uint64_t>(rows) * t) / threads);
  }
  for (std::uint32_t t = 0; t < threads; ++t) {
    gather_rows(fmt, payload, meta, cols, begins[t], begins[t + 1], ps[t], ms[t]);
    stages.push_back(make_stage(fmt, begins[t + 1] - begins[t], cols));
  }
  const std::vector<float> act(activation, activation + cols);
  std::vector<std::vector<float>> results(threads);
  const auto start = std::chrono::steady_clock::now();
  std::vector<std::thread> pool;
  for (std::uint32_t t = 0; t < threads; ++t) {
    pool.emplace_back([&, t] { results[t] = reference_stage_logits(stages[t], ps[t], ms[t], act); });
  }
  for (auto& th : pool) th.join();
  const auto stop = std::chrono::steady_clock::now();
  if (out != nullptr) {
    for (std::uint32_t t = 0; t < threads; ++t) {
      std::memcpy(out + begins[t], results[t].data(), results[t].size() * sizeof(float));
    }
  }
  return std::chrono::duration<double>(stop - start).count();
}

}  // extern "C"
