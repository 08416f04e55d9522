/*
 * qoracle.c -- CPU restatement of the reference's decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * local-ai-gpu-acceleration_b200/csrc; only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load it.  The product path
 * never calls it and has no CPU fallback.
 *
 * Every function restates one function of the reference (MKKSANDI/local-ai-gpu-
 * acceleration) and cites it as path:line.  Arithmetic is written in the same
 * order as the reference and the file is compiled with -ffp-contract=off so the
 * host compiler cannot fuse a multiply and an add the reference keeps separate.
 *
 * Parity pin: tests/test_oracle_cpu.py checks these functions bit-for-bit against
 * tests/golden/*.npz, which tests/golden/make_golden.py produced by calling the
 * reference's own CPU functions (runtime/apps/mixed_sequence_benchmark_runner/
 * main.cpp:1086-1341, compiled unmodified by oracle/Makefile into oracle/_ref).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "../include/qgemv_b200.h"
#include "../local-ai-gpu-acceleration_b200/csrc/iq_grids.h"

static const uint16_t k_iq2s_kgrid[1024] = {QG_IQ2S_KGRID_VALUES};
static const uint32_t k_iq3s_grid[512] = {QG_IQ3S_GRID_VALUES};

/* runtime/apps/mixed_sequence_benchmark_runner/main.cpp:1086-1098 (device twin
 * runtime/kernels/decode/decode_kernels.cu:1665-1676). */
float orc_fp16_to_f32(uint16_t bits) {
  const float sign = (bits & 0x8000u) ? -1.0f : 1.0f;
  const int exp = (int)((bits >> 10u) & 0x1fu);
  const int mant = (int)(bits & 0x03ffu);
  if (exp == 0) {
    return mant == 0 ? sign * 0.0f : sign * ldexpf((float)mant, -24);
  }
  if (exp == 31) {
    return mant == 0 ? sign * INFINITY : NAN;
  }
  return sign * ldexpf(1.0f + (float)mant / 1024.0f, exp - 15);
}

static uint16_t rd_u16(const uint8_t* p) { return (uint16_t)(p[0] | ((uint16_t)p[1] << 8u)); }

static float rd_f32(const uint8_t* p) {
  float v;
  memcpy(&v, p, sizeof v);
  return v;
}

/* main.cpp:1100-1114; decode_kernels.cu:1678-1692; tools/bench/q4k_resident_pack.py:52-57 */
void orc_scale_min_k4(int index, const uint8_t* packed, uint8_t* scale, uint8_t* min_value) {
  if (index < 4) {
    *scale = (uint8_t)(packed[index] & 63u);
    *min_value = (uint8_t)(packed[index + 4] & 63u);
    return;
  }
  *scale = (uint8_t)((packed[index + 4] & 0x0fu) | ((packed[index - 4] >> 6u) << 4u));
  *min_value = (uint8_t)((packed[index + 4] >> 4u) | ((packed[index] >> 6u) << 4u));
}

/* Q4_K split packs: main.cpp:1133-1171 (q4k_dequant_value).  The raw 144-B block is
 * the split-native case with meta = block[0:16] and payload = block[16:144]
 * (tools/bench/q4k_resident_pack.py:104-106,141-145; second oracle:
 * runtime/apps/fused_benchmark_runner/main.cpp:871-909, same arithmetic). */
static float q4k_dequant(const uint8_t* payload_block, const uint8_t* meta, int fmt,
                         uint32_t value_index) {
  const uint32_t group64 = value_index >> 6u;
  const uint32_t within64 = value_index & 63u;
  const uint32_t lane = within64 & 31u;
  const int high_half = within64 >= 32u;
  const uint32_t pair = group64 * 2u + (high_half ? 1u : 0u);
  const uint8_t packed = payload_block[group64 * 32u + lane];
  const float quant = (float)(high_half ? (packed >> 4u) : (packed & 0x0fu));
  switch (fmt) {
    case QG_FMT_Q4K_SPLIT_PREDECODED: {
      const uint8_t* pm = meta + pair * 2u * 4u;
      return rd_f32(pm) * quant - rd_f32(pm + 4);
    }
    case QG_FMT_Q4K_SPLIT_HALF: {
      const uint8_t* pm = meta + pair * 2u * 2u;
      return orc_fp16_to_f32(rd_u16(pm)) * quant - orc_fp16_to_f32(rd_u16(pm + 2));
    }
    case QG_FMT_Q4K_SPLIT_COMPACT: {
      const float d = orc_fp16_to_f32(rd_u16(meta));
      const float dmin = orc_fp16_to_f32(rd_u16(meta + 2));
      return d * (float)meta[4u + pair] * quant - dmin * (float)meta[12u + pair];
    }
    default: { /* QG_FMT_Q4K_RAW and QG_FMT_Q4K_SPLIT_NATIVE */
      const float d = orc_fp16_to_f32(rd_u16(meta));
      const float dmin = orc_fp16_to_f32(rd_u16(meta + 2));
      uint8_t sc = 0, mn = 0;
      orc_scale_min_k4((int)pair, meta + 4, &sc, &mn);
      return d * (float)sc * quant - dmin * (float)mn;
    }
  }
}

/* main.cpp:1231-1259 (device twin decode_kernels.cu:1694-1728). */
static float q5k_dequant(const uint8_t* block, uint32_t value_index) {
  const float d = orc_fp16_to_f32(rd_u16(block + 0));
  const float dmin = orc_fp16_to_f32(rd_u16(block + 2));
  const uint8_t* scales = block + 4;
  const uint8_t* qh = block + 16;
  const uint8_t* qs = block + 48;
  const uint32_t group64 = value_index >> 6u;
  const uint32_t within64 = value_index & 63u;
  const uint32_t lane = within64 & 31u;
  const int high_half = within64 >= 32u;
  const uint32_t scale_index = group64 * 2u + (high_half ? 1u : 0u);
  uint8_t sc = 0, mn = 0;
  orc_scale_min_k4((int)scale_index, scales, &sc, &mn);
  const uint8_t packed = qs[group64 * 32u + lane];
  const uint8_t low_bits = high_half ? (uint8_t)(packed >> 4u) : (uint8_t)(packed & 0x0fu);
  const uint8_t high_mask = (uint8_t)((high_half ? 2u : 1u) << (group64 * 2u));
  const uint8_t quant = (uint8_t)(low_bits + ((qh[lane] & high_mask) ? 16u : 0u));
  return d * (float)sc * (float)quant - dmin * (float)mn;
}

/* main.cpp:1173-1194 (device twin decode_kernels.cu:1504-1527). */
static float iq2s_dequant(const uint8_t* block, uint32_t value_index) {
  const uint32_t ib32 = value_index >> 5u;
  const uint32_t within32 = value_index & 31u;
  const uint32_t group = within32 >> 3u;
  const uint32_t lane = within32 & 7u;
  const float d = orc_fp16_to_f32(rd_u16(block));
  const uint8_t* qs = block + 2;
  const uint8_t* qh = block + 66;
  const uint8_t* scales = block + 74;
  const uint32_t group_offset = ib32 * 4u + group;
  const uint32_t grid_index =
      qs[group_offset] | (((uint32_t)qh[ib32] << (8u - 2u * group)) & 0x300u);
  const uint32_t packed_grid = k_iq2s_kgrid[grid_index];
  const uint32_t grid = 2u * ((packed_grid >> (2u * lane)) & 0x3u) + 1u;
  const uint32_t scale_nibble = group < 2u ? (scales[ib32] & 0x0fu) : (scales[ib32] >> 4u);
  const float scale = d * (0.5f + (float)scale_nibble) * 0.25f;
  const int negative = (qs[32u + group_offset] & (1u << lane)) != 0u;
  return scale * (float)grid * (negative ? -1.0f : 1.0f);
}

/* main.cpp:1196-1221 (device twin decode_kernels.cu:1529-1557). */
static float iq3s_dequant(const uint8_t* block, uint32_t value_index) {
  const uint32_t ib32 = value_index >> 5u;
  const uint32_t within32 = value_index & 31u;
  const uint32_t group = within32 >> 3u;
  const uint32_t lane = within32 & 7u;
  const uint32_t pair = lane >> 2u;
  const uint32_t grid_lane = lane & 3u;
  const float d = orc_fp16_to_f32(rd_u16(block));
  const uint8_t* qs = block + 2;
  const uint8_t* qh = block + 66;
  const uint8_t* signs = block + 74;
  const uint8_t* scales = block + 106;
  const uint32_t selector_index = ib32 * 8u + group * 2u + pair;
  const uint32_t high_bit = (qh[ib32] >> (2u * group + pair)) & 1u;
  const uint32_t grid_index = qs[selector_index] | (high_bit << 8u);
  const uint32_t packed_grid = k_iq3s_grid[grid_index];
  const uint32_t grid = (packed_grid >> (8u * grid_lane)) & 0xffu;
  const uint32_t scale_nibble =
      (ib32 & 1u) == 0u ? (scales[ib32 >> 1u] & 0x0fu) : (scales[ib32 >> 1u] >> 4u);
  const float scale = d * (float)(1u + 2u * scale_nibble);
  const int negative = (signs[ib32 * 4u + group] & (1u << lane)) != 0u;
  return scale * (float)grid * (negative ? -1.0f : 1.0f);
}

/* Dequantize value `value_index` (0..255) of super-block `block_index` (row-major
 * block order) of a pack.  For Q4_K split formats `payload` is the 128-B/blk stream
 * and `meta` the side table; for every other format `meta` is unused. */
float orc_dequant_value(int fmt, const uint8_t* payload, const uint8_t* meta,
                        uint64_t block_index, uint32_t value_index) {
  switch (fmt) {
    case QG_FMT_Q4K_RAW: {
      const uint8_t* blk = payload + block_index * 144u;
      return q4k_dequant(blk + 16, blk, fmt, value_index);
    }
    case QG_FMT_Q4K_SPLIT_PREDECODED:
    case QG_FMT_Q4K_SPLIT_HALF:
    case QG_FMT_Q4K_SPLIT_COMPACT:
    case QG_FMT_Q4K_SPLIT_NATIVE:
      return q4k_dequant(payload + block_index * 128u,
                         meta + block_index * qg_meta_bytes_per_block(fmt), fmt, value_index);
    case QG_FMT_Q5K:
      return q5k_dequant(payload + block_index * 176u, value_index);
    case QG_FMT_IQ2S:
      return iq2s_dequant(payload + block_index * 82u, value_index);
    case QG_FMT_IQ3S:
      return iq3s_dequant(payload + block_index * 110u, value_index);
    default:
      return NAN;
  }
}

/* Dequantize `block_count` whole super-blocks into out[block_count*256]. */
void orc_dequant_blocks(int fmt, const uint8_t* payload, const uint8_t* meta,
                        uint64_t first_block, uint64_t block_count, float* out) {
  for (uint64_t b = 0; b < block_count; ++b) {
    for (uint32_t v = 0; v < 256u; ++v) {
      out[b * 256u + v] = orc_dequant_value(fmt, payload, meta, first_block + b, v);
    }
  }
}

/* reference_stage_logits, main.cpp:1262-1309: sequential fp32 accumulation over
 * the columns of each row, value by value.  Rows [row_begin, row_end) only. */
void orc_matvec_rows(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                     uint32_t cols, uint32_t row_begin, uint32_t row_end, float* y) {
  const uint32_t bpr = cols / 256u;
  for (uint32_t row = row_begin; row < row_end; ++row) {
    float acc = 0.0f;
    for (uint32_t col = 0; col < cols; ++col) {
      const uint64_t bi = (uint64_t)row * bpr + col / 256u;
      acc += orc_dequant_value(fmt, payload, meta, bi, col & 255u) * x[col];
    }
    y[row - row_begin] = acc;
  }
}

void orc_matvec(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                uint32_t rows, uint32_t cols, float* y) {
  orc_matvec_rows(fmt, payload, meta, x, cols, 0, rows, y);
}

/* Batched: Y[b, r] = sum_c W[r, c] X[b, c], each (b, r) accumulated like the
 * batch-1 reference.  No reference counterpart (all reference kernels are batch 1). */
void orc_matvec_batched(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                        uint32_t batch, uint32_t rows, uint32_t cols, float* y) {
  for (uint32_t b = 0; b < batch; ++b) {
    orc_matvec(fmt, payload, meta, x + (uint64_t)b * cols, rows, cols, y + (uint64_t)b * rows);
  }
}

/* Row L1 norms sum_c |W[r, c]| -- used to state the matvec tolerance
 * 1e-3 * ||w_row||_1 * ||x||_inf. */
void orc_row_l1(int fmt, const uint8_t* payload, const uint8_t* meta, uint32_t rows,
                uint32_t cols, float* out) {
  const uint32_t bpr = cols / 256u;
  for (uint32_t row = 0; row < rows; ++row) {
    double acc = 0.0;
    for (uint32_t col = 0; col < cols; ++col) {
      acc += fabs((double)orc_dequant_value(fmt, payload, meta, (uint64_t)row * bpr + col / 256u,
                                            col & 255u));
    }
    out[row] = (float)acc;
  }
}

/* main.cpp:1311-1322 (argmax_token) -- lowest index wins ties. */
uint32_t orc_argmax(const float* logits, uint32_t n) {
  float best_value = -3.4028234663852886e38f;
  uint32_t best_index = 0;
  for (uint32_t row = 0; row < n; ++row) {
    const float value = logits[row];
    if (value > best_value || (value == best_value && row < best_index)) {
      best_value = value;
      best_index = row;
    }
  }
  return best_index;
}

/* main.cpp:1324-1341 (apply_reference_kv): KV page write with the pre-update token. */
void orc_apply_kv(const float* logits, uint32_t rows, float* kv, uint64_t kv_words,
                  uint32_t token, uint32_t page_words, uint32_t active_pages) {
  if (kv_words == 0 || page_words == 0u) return;
  const uint32_t active_rows = rows < active_pages ? rows : active_pages;
  for (uint32_t row = 0; row < active_rows; ++row) {
    const uint64_t page_base = (uint64_t)row * page_words;
    const uint64_t offset = (uint64_t)((token + row) % page_words);
    kv[(page_base + offset) % kv_words] = logits[row];
  }
}

/* One matvec stage of the reference launchers (decode_kernels.cu:4032-4177,
 * 4609-4639) as the mixed runner's reference replays it (main.cpp:2729-2735):
 * logits, KV write with the pre-update token, then token = (argmax+token+1)%32000. */
void orc_decode_stage(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                      uint32_t rows, uint32_t cols, float* logits, float* kv, uint64_t kv_words,
                      uint32_t* token, uint32_t page_words, uint32_t active_pages) {
  orc_matvec(fmt, payload, meta, x, rows, cols, logits);
  orc_apply_kv(logits, rows, kv, kv_words, *token, page_words, active_pages);
  *token = (orc_argmax(logits, rows) + *token + 1u) % 32000u;
}

/* decode_kernels.cu:3033-3073 (output_token_sample_kernel). */
uint32_t orc_output_token_sample(const float* logits, uint32_t rows, uint32_t vocab_size,
                                 uint32_t token_offset) {
  return (orc_argmax(logits, rows) + token_offset) % vocab_size;
}

/* ---- feedback kernels of the mixed runner (main.cpp:1362-1500; device kernels
 * decode_kernels.cu:122-289).  All share the unweighted RMS of logits[0:rows]. */
static float inv_rms_of(const float* logits, uint32_t rows, float eps) {
  float sum_sq = 0.0f;
  for (uint32_t r = 0; r < rows; ++r) sum_sq += logits[r] * logits[r];
  const float mean_sq = sum_sq / (float)rows;
  return 1.0f / sqrtf(mean_sq + eps);
}

static float silu_f(float v) { return v * (1.0f / (1.0f + expf(-v))); }

/* decode_kernels.cu:122-141; main.cpp:1362-1381 */
void orc_rmsnorm_feedback(const float* logits, float* act, uint32_t rows, uint32_t cols,
                          float eps) {
  if (rows == 0) return;
  const float inv = inv_rms_of(logits, rows, eps);
  for (uint32_t c = 0; c < cols; ++c) act[c] = logits[c % rows] * inv;
}

/* decode_kernels.cu:143-164; main.cpp:1383-1403 */
void orc_silu_rmsnorm_feedback(const float* logits, float* act, uint32_t rows, uint32_t cols,
                               float eps) {
  if (rows == 0) return;
  const float inv = inv_rms_of(logits, rows, eps);
  for (uint32_t c = 0; c < cols; ++c) act[c] = silu_f(logits[c % rows] * inv);
}

/* decode_kernels.cu:166-189; main.cpp:1405-1430 */
void orc_rmsnorm_feedback_with_silu_cache(const float* logits, float* act, float* silu_cache,
                                          uint32_t rows, uint32_t cols, float eps) {
  if (rows == 0) return;
  const float inv = inv_rms_of(logits, rows, eps);
  for (uint32_t c = 0; c < cols; ++c) {
    const float n = logits[c % rows] * inv;
    act[c] = n;
    silu_cache[c] = silu_f(n);
  }
}

/* decode_kernels.cu:191-213; main.cpp:1432-1452 */
void orc_gated_silu_rmsnorm_feedback(const float* logits, const float* silu_cache, float* act,
                                     uint32_t rows, uint32_t cache_cols, uint32_t cols,
                                     float eps) {
  if (rows == 0 || cache_cols == 0) return;
  const float inv = inv_rms_of(logits, rows, eps);
  for (uint32_t c = 0; c < cols; ++c) act[c] = silu_cache[c % cache_cols] * (logits[c % rows] * inv);
}

/* decode_kernels.cu:215-238 (silu=1) and 240-261 (silu=0); main.cpp:1454-1480 */
void orc_rmsnorm_cache(const float* logits, float* cache, uint32_t rows, uint32_t cache_cols,
                       float eps, int apply_silu, int accumulate) {
  if (rows == 0) return;
  const float inv = inv_rms_of(logits, rows, eps);
  for (uint32_t c = 0; c < cache_cols; ++c) {
    float v = logits[c % rows] * inv;
    if (apply_silu) v = silu_f(v);
    cache[c] = accumulate ? cache[c] + v : v;
  }
}

/* decode_kernels.cu:263-289 */
void orc_rmsnorm_cache_and_gated_product(const float* logits, const float* gate_cache,
                                         float* up_cache, float* act, uint32_t rows,
                                         uint32_t cache_cols, uint32_t output_cols, float eps,
                                         int accumulate) {
  if (rows == 0 || cache_cols == 0) return;
  const float inv = inv_rms_of(logits, rows, eps);
  for (uint32_t c = 0; c < output_cols; ++c) {
    const float v = logits[c % rows] * inv;
    const float up = accumulate ? up_cache[c] + v : v;
    up_cache[c] = up;
    act[c] = gate_cache[c] * up;
  }
}

/* ---- Llama-style layer-slice math with no reference counterpart (the reference's
 * RMSNorm is unweighted and its attention is a passthrough:
 * main.cpp:195, decode_kernels.cu:122-141).  Plain restatements used as the
 * checker for the fused epilogues. */

/* y = x / sqrt(mean(x^2) + eps) * w */
void orc_weighted_rmsnorm(const float* x, const float* w, uint32_t n, float eps, float* y) {
  float sum_sq = 0.0f;
  for (uint32_t i = 0; i < n; ++i) sum_sq += x[i] * x[i];
  const float inv = 1.0f / sqrtf(sum_sq / (float)n + eps);
  for (uint32_t i = 0; i < n; ++i) y[i] = x[i] * inv * w[i];
}

/* h = silu(gate) * up */
void orc_silu_gate(const float* gate, const float* up, uint32_t n, float* h) {
  for (uint32_t i = 0; i < n; ++i) h[i] = silu_f(gate[i]) * up[i];
}

/* out = a + b */
void orc_residual_add(const float* a, const float* b, uint32_t n, float* out) {
  for (uint32_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}
