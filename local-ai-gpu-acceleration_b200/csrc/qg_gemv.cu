// qg_gemv.cu -- batch-1 quantized GEMV for sm_100a (the decode hot path).
//
// Design (one kernel per pack format, template FMT):
//  * Persistent CTAs (grid = min(tiles, SMs x resident CTAs)).  A tile is a run of
//    consecutive rows; its bytes are contiguous in the pack (payload and, for
//    Q4_K split packs, metadata), so one elected thread streams each tile into a
//    shared-memory ring of S stages with 1-D TMA (cp.async.bulk, mbarrier
//    completion, L2 evict-first) while the other threads decode the previous ones.
//  * Thread (slot, c) owns the 64-column chunk c of one row of every pass; it
//    loads x[64c .. 64c+64) into registers once, so x is never re-read from
//    memory, and each thread reads only the 32-48 B of its chunk from shared
//    memory per row.
//  * Row sums: shuffle reduction inside aligned lane groups of gcd(cols/64, 32),
//    then one shared-memory pass per tile; the epilogue writes y (+ residual) and
//    the reference's KV page word.
//  * Every mbarrier wait is bounded (QG_ERR_WAIT_TIMEOUT); tiles whose byte count
//    or address cannot go through TMA are copied by all threads instead.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "iq_grids.h"
#include "qg_formats.cuh"
#include "qg_host.h"

namespace qg {

__device__ unsigned int g_error_word = 0u;
__device__ uint16_t g_iq2s_kgrid[1024] = {QG_IQ2S_KGRID_VALUES};
__device__ uint32_t g_iq3s_grid[512] = {QG_IQ3S_GRID_VALUES};

struct GemvArgs {
  const uint8_t* payload;
  const uint8_t* meta;
  const float* x;
  float* y;
  const float* residual;  // optional: y = residual + W x
  float* kv;              // optional KV page write (reference epilogue)
  const uint32_t* token;
  uint64_t kv_words;
  uint32_t page_words;
  uint32_t active_pages;
  uint32_t rows;
  uint32_t cols;
  uint32_t tpr;           // threads per row = cols / 64
  uint32_t group;         // shuffle-reduction group = gcd(tpr, 32)
  uint32_t rpp;           // rows per pass
  uint32_t passes;        // passes per tile
  uint32_t rows_per_tile;
  uint32_t num_tiles;
  uint32_t stages;
  uint32_t stage_bytes;   // payload + metadata of one tile, 128-B multiple
  uint32_t meta_off;      // metadata offset inside a stage
  uint32_t red_off;       // reduction buffer offset in dynamic smem
  uint32_t table_off;     // codebook offset in dynamic smem
  uint32_t stage_off;     // first stage offset in dynamic smem
  uint32_t tma_ok;        // base pointers 16-B aligned and full tiles 16-B multiples
};

template <int FMT>
__device__ __forceinline__ void issue_tile(const GemvArgs& a, uint8_t* stage, uint64_t* bar,
                                           uint32_t tile, uint64_t policy) {
  constexpr uint32_t PB = FmtTraits<FMT>::payload_bytes;
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  const uint32_t bpr = a.cols >> 8;
  const uint32_t row0 = tile * a.rows_per_tile;
  const uint32_t nrows = min(a.rows_per_tile, a.rows - row0);
  const uint32_t pb = nrows * bpr * PB;
  const uint32_t mb = nrows * bpr * MB;
  mbar_arrive_expect_tx(bar, pb + mb);
  tma_load_1d(stage, a.payload + static_cast<uint64_t>(row0) * bpr * PB, pb, bar, policy);
  if (MB != 0u) {
    tma_load_1d(stage + a.meta_off, a.meta + static_cast<uint64_t>(row0) * bpr * MB, mb, bar,
                policy);
  }
}

template <int FMT>
__device__ __forceinline__ bool tile_via_tma(const GemvArgs& a, uint32_t tile) {
  constexpr uint32_t PB = FmtTraits<FMT>::payload_bytes;
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  if (!a.tma_ok) return false;
  const uint32_t bpr = a.cols >> 8;
  const uint32_t nrows = min(a.rows_per_tile, a.rows - tile * a.rows_per_tile);
  return ((nrows * bpr * PB) & 15u) == 0u && ((nrows * bpr * MB) & 15u) == 0u;
}

template <int FMT>
__global__ void __launch_bounds__(512, 1) gemv_kernel(const GemvArgs a) {
  constexpr uint32_t PB = FmtTraits<FMT>::payload_bytes;
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  float* red = reinterpret_cast<float*>(smem + a.red_off);
  uint8_t* stages = smem + a.stage_off;
  uint16_t* kgrid = reinterpret_cast<uint16_t*>(smem + a.table_off);
  uint32_t* grid3 = reinterpret_cast<uint32_t*>(smem + a.table_off);

  const uint32_t tid = threadIdx.x;
  const uint32_t nthreads = blockDim.x;
  const bool valid = tid < a.rpp * a.tpr;
  const uint32_t slot = valid ? tid / a.tpr : 0u;
  const uint32_t c = valid ? tid - slot * a.tpr : 0u;
  const uint32_t bpr = a.cols >> 8;
  const uint32_t groups_per_row = a.tpr / a.group;

  const uint32_t first = blockIdx.x, stride = gridDim.x;
  const uint32_t n_my = a.num_tiles > first ? (a.num_tiles - first + stride - 1u) / stride : 0u;

  uint64_t policy = 0;
  if (tid == 0u) {
    policy = l2_evict_first_policy();
    for (uint32_t s = 0; s < a.stages; ++s) mbar_init(&bars[s], 1u);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0u) {
    const uint32_t pro = min(a.stages, n_my);
    for (uint32_t i = 0; i < pro; ++i) {
      const uint32_t tile = first + i * stride;
      if (tile_via_tma<FMT>(a, tile)) {
        issue_tile<FMT>(a, stages + i * a.stage_bytes, &bars[i], tile, policy);
      }
    }
  }

  // Codebooks into shared memory (overlaps the first TMA loads).
  if (FMT == QG_FMT_IQ2S) {
    for (uint32_t i = tid; i < 1024u; i += nthreads) kgrid[i] = g_iq2s_kgrid[i];
  } else if (FMT == QG_FMT_IQ3S) {
    for (uint32_t i = tid; i < 512u; i += nthreads) grid3[i] = g_iq3s_grid[i];
  }

  // This thread's 64 x values and their two 32-value sums.
  ChunkX xr;
  {
    const float* xp = a.x + 64u * c;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      xr.a[i] = make_float2(__ldg(xp + 2 * i), __ldg(xp + 2 * i + 1));
      xr.b[i] = make_float2(__ldg(xp + 32 + 2 * i), __ldg(xp + 33 + 2 * i));
    }
    float sa = 0.f, sb = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      sa += xr.a[i].x + xr.a[i].y;
      sb += xr.b[i].x + xr.b[i].y;
    }
    xr.sa = sa;
    xr.sb = sb;
  }
  const uint32_t tok = (a.kv != nullptr && a.token != nullptr) ? *a.token : 0u;
  __syncthreads();  // codebooks visible

  uint32_t phase_bits = 0u;
  bool failed = false;
  for (uint32_t i = 0; i < n_my; ++i) {
    const uint32_t tile = first + i * stride;
    const uint32_t s = i % a.stages;
    uint8_t* st = stages + s * a.stage_bytes;
    const uint32_t row0 = tile * a.rows_per_tile;
    const uint32_t nrows = min(a.rows_per_tile, a.rows - row0);
    if (tile_via_tma<FMT>(a, tile)) {
      if (!mbar_wait_bounded(&bars[s], (phase_bits >> s) & 1u)) failed = true;
      phase_bits ^= 1u << s;
    } else {
      // All-thread byte copy (unaligned base or a tail tile whose size is not a
      // 16-B multiple).
      const uint64_t pbytes = static_cast<uint64_t>(nrows) * bpr * PB;
      const uint8_t* src = a.payload + static_cast<uint64_t>(row0) * bpr * PB;
      for (uint64_t o = tid; o < pbytes; o += nthreads) st[o] = src[o];
      if (MB != 0u) {
        const uint64_t mbytes = static_cast<uint64_t>(nrows) * bpr * MB;
        const uint8_t* msrc = a.meta + static_cast<uint64_t>(row0) * bpr * MB;
        for (uint64_t o = tid; o < mbytes; o += nthreads) st[a.meta_off + o] = msrc[o];
      }
      __syncthreads();
    }
    if (__syncthreads_or(failed)) break;

    float* rb = red + (i & 1u) * (a.rows_per_tile * groups_per_row);
    for (uint32_t p = 0; p < a.passes; ++p) {
      const uint32_t lr = p * a.rpp + slot;
      float part = 0.f;
      if (valid && lr < nrows) {
        const uint8_t* rp = st + static_cast<uint64_t>(lr) * bpr * PB;
        const uint8_t* rm = st + a.meta_off + static_cast<uint64_t>(lr) * bpr * MB;
        part = chunk_dot<FMT>(rp, rm, c, xr, kgrid, grid3);
      }
      for (uint32_t off = a.group >> 1; off > 0u; off >>= 1) {
        part += __shfl_xor_sync(0xffffffffu, part, off);
      }
      if (valid && lr < nrows && (c % a.group) == 0u) {
        rb[lr * groups_per_row + c / a.group] = part;
      }
    }
    __syncthreads();  // stage s fully read; row partials complete
    if (tid == 0u && i + a.stages < n_my) {
      const uint32_t nt = first + (i + a.stages) * stride;
      if (tile_via_tma<FMT>(a, nt)) {
        fence_proxy_async_smem();
        issue_tile<FMT>(a, st, &bars[s], nt, policy);
      }
    }
    for (uint32_t t = tid; t < nrows; t += nthreads) {
      float v = 0.f;
      for (uint32_t q = 0; q < groups_per_row; ++q) v += rb[t * groups_per_row + q];
      const uint32_t row = row0 + t;
      if (a.residual != nullptr) v += a.residual[row];
      a.y[row] = v;
      if (a.kv != nullptr && row < a.active_pages && a.kv_words > 0u && a.page_words > 0u) {
        const uint64_t base = static_cast<uint64_t>(row) * a.page_words;
        const uint64_t off = (tok + row) % a.page_words;
        a.kv[(base + off) % a.kv_words] = v;
      }
    }
  }
  if (failed && tid == 0u) {
    // Give copies still in flight a bounded chance to land before the CTA exits.
    for (uint32_t k = 0; k < a.stages; ++k) mbar_wait_bounded(&bars[k], (phase_bits >> k) & 1u);
  }
}

// Shapes the tiled kernel does not take (cols/64 > 512): one CTA per row, values
// decoded one at a time.  Correct for every shape, not tuned.
template <int FMT>
__global__ void __launch_bounds__(256) gemv_rowwise_kernel(const GemvArgs a) {
  __shared__ float part[256];
  const uint32_t row = blockIdx.x;
  if (row >= a.rows) return;
  const uint32_t bpr = a.cols >> 8;
  float acc = 0.f;
  for (uint32_t col = threadIdx.x; col < a.cols; col += blockDim.x) {
    acc += dequant_value<FMT>(a.payload, a.meta, static_cast<uint64_t>(row) * bpr + (col >> 8),
                              col & 255u) *
           a.x[col];
  }
  part[threadIdx.x] = acc;
  __syncthreads();
  for (uint32_t s = blockDim.x / 2u; s > 0u; s >>= 1) {
    if (threadIdx.x < s) part[threadIdx.x] += part[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0u) {
    float v = part[0];
    if (a.residual != nullptr) v += a.residual[row];
    a.y[row] = v;
    if (a.kv != nullptr && a.token != nullptr && row < a.active_pages && a.kv_words > 0u &&
        a.page_words > 0u) {
      const uint64_t base = static_cast<uint64_t>(row) * a.page_words;
      const uint64_t off = (*a.token + row) % a.page_words;
      a.kv[(base + off) % a.kv_words] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Host-side planning and launch.

namespace {

uint32_t gcd_u32(uint32_t a, uint32_t b) {
  while (b != 0u) {
    const uint32_t t = a % b;
    a = b;
    b = t;
  }
  return a;
}

struct DeviceInfo {
  int sms = 0;
  int max_smem_optin = 0;
};

DeviceInfo device_info() {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return DeviceInfo{148, 227 * 1024};
  if (cache[dev].sms == 0) {
    cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  }
  return cache[dev];
}

template <int FMT>
cudaError_t launch_gemv_fmt(GemvArgs a, cudaStream_t stream) {
  constexpr uint32_t PB = FmtTraits<FMT>::payload_bytes;
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  const DeviceInfo dev = device_info();
  const uint32_t bpr = a.cols >> 8;
  a.tpr = a.cols / 64u;
  if (a.cols < 256u || a.tpr > 512u) {
    gemv_rowwise_kernel<FMT><<<a.rows, 256, 0, stream>>>(a);
    return cudaGetLastError();
  }
  GemvPlan plan = plan_gemv(FMT, a.rows, a.cols, dev.sms);
  if (plan.smem_bytes > static_cast<uint32_t>(dev.max_smem_optin)) {
    gemv_rowwise_kernel<FMT><<<a.rows, 256, 0, stream>>>(a);
    return cudaGetLastError();
  }
  a.group = plan.group;
  a.rpp = plan.rpp;
  a.passes = plan.passes;
  a.rows_per_tile = plan.rows_per_tile;
  a.num_tiles = plan.num_tiles;
  a.stages = plan.stages;
  a.stage_bytes = plan.stage_bytes;
  a.meta_off = plan.meta_off;
  a.red_off = plan.red_off;
  a.table_off = plan.table_off;
  a.stage_off = plan.stage_off;
  const bool aligned = (reinterpret_cast<uintptr_t>(a.payload) & 15u) == 0u &&
                       (MB == 0u || (reinterpret_cast<uintptr_t>(a.meta) & 15u) == 0u);
  a.tma_ok = (aligned && ((a.rows_per_tile * bpr * PB) & 15u) == 0u &&
              ((a.rows_per_tile * bpr * MB) & 15u) == 0u)
                 ? 1u
                 : 0u;
  const size_t smem = plan.smem_bytes;
  static thread_local int configured[64][QG_FMT_COUNT] = {};
  int devid = 0;
  cudaGetDevice(&devid);
  if (devid >= 0 && devid < 64 && configured[devid][FMT] < static_cast<int>(smem)) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<FMT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         dev.max_smem_optin);
    if (e != cudaSuccess) return e;
    configured[devid][FMT] = dev.max_smem_optin;
  }
  gemv_kernel<FMT><<<plan.grid, plan.threads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

GemvPlan plan_gemv(int fmt, uint32_t rows, uint32_t cols, int sms) {
  GemvPlan p{};
  const uint32_t PB = qg_payload_bytes_per_block(fmt);
  const uint32_t MB = qg_meta_bytes_per_block(fmt);
  const uint32_t bpr = cols >> 8;
  const uint32_t tpr = cols / 64u;
  p.group = gcd_u32(tpr, 32u);
  // Smallest rows-per-pass whose thread count is a whole number of warps, then as
  // many as fit in ~256 threads.
  const uint32_t base = 32u / p.group;
  uint32_t rpp = base;
  if (rpp * tpr > 512u) rpp = 1u;  // pad the last warp with idle threads
  while ((rpp + base) * tpr <= 256u) rpp += base;
  p.rpp = rpp;
  p.threads = ((rpp * tpr + 31u) / 32u) * 32u;
  const uint32_t row_bytes = bpr * PB, row_meta = bpr * MB;
  // ~16 KB of payload per tile, at most 4 passes.
  uint32_t passes = std::max(1u, std::min(4u, 16384u / std::max(1u, rpp * row_bytes)));
  // Full tiles must be 16-B multiples to go through TMA.
  for (uint32_t k = passes; k <= passes * 16u; ++k) {
    if (((k * rpp * row_bytes) & 15u) == 0u && ((k * rpp * row_meta) & 15u) == 0u) {
      passes = k;
      break;
    }
  }
  p.passes = passes;
  p.rows_per_tile = passes * rpp;
  p.num_tiles = (rows + p.rows_per_tile - 1u) / p.rows_per_tile;
  const uint32_t pay = p.rows_per_tile * row_bytes, met = p.rows_per_tile * row_meta;
  p.meta_off = (pay + 127u) & ~127u;
  p.stage_bytes = (p.meta_off + met + 127u) & ~127u;
  if (MB == 0u) p.stage_bytes = (pay + 127u) & ~127u;
  const uint32_t budget = 96u * 1024u;
  p.stages = std::max(2u, std::min(8u, budget / p.stage_bytes));
  const uint32_t red_floats = 2u * p.rows_per_tile * (tpr / p.group);
  p.red_off = 128u;
  p.table_off = (p.red_off + red_floats * 4u + 127u) & ~127u;
  const uint32_t table_bytes = (fmt == QG_FMT_IQ2S || fmt == QG_FMT_IQ3S) ? 2048u : 0u;
  p.stage_off = (p.table_off + table_bytes + 127u) & ~127u;
  p.smem_bytes = p.stage_off + p.stages * p.stage_bytes;
  const uint32_t by_smem = std::max(1u, (228u * 1024u) / (p.smem_bytes + 1024u));
  const uint32_t by_threads = std::max(1u, 2048u / p.threads);
  const uint32_t by_regs = std::max(1u, 65536u / (p.threads * 128u));
  const uint32_t per_sm = std::min(by_smem, std::min(by_threads, by_regs));
  p.grid = std::min(p.num_tiles, static_cast<uint32_t>(sms) * per_sm);
  if (p.grid == 0u) p.grid = 1u;
  return p;
}

cudaError_t launch_gemv(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                        float* y, const float* residual, float* kv, const uint32_t* token,
                        uint64_t kv_words, uint32_t page_words, uint32_t active_pages,
                        uint32_t rows, uint32_t cols, cudaStream_t stream) {
  GemvArgs a{};
  a.payload = payload;
  a.meta = meta;
  a.x = x;
  a.y = y;
  a.residual = residual;
  a.kv = kv;
  a.token = token;
  a.kv_words = kv_words;
  a.page_words = page_words;
  a.active_pages = active_pages;
  a.rows = rows;
  a.cols = cols;
  switch (fmt) {
    case QG_FMT_Q4K_RAW: return launch_gemv_fmt<QG_FMT_Q4K_RAW>(a, stream);
    case QG_FMT_Q4K_SPLIT_PREDECODED: return launch_gemv_fmt<QG_FMT_Q4K_SPLIT_PREDECODED>(a, stream);
    case QG_FMT_Q4K_SPLIT_HALF: return launch_gemv_fmt<QG_FMT_Q4K_SPLIT_HALF>(a, stream);
    case QG_FMT_Q4K_SPLIT_COMPACT: return launch_gemv_fmt<QG_FMT_Q4K_SPLIT_COMPACT>(a, stream);
    case QG_FMT_Q4K_SPLIT_NATIVE: return launch_gemv_fmt<QG_FMT_Q4K_SPLIT_NATIVE>(a, stream);
    case QG_FMT_Q5K: return launch_gemv_fmt<QG_FMT_Q5K>(a, stream);
    case QG_FMT_IQ2S: return launch_gemv_fmt<QG_FMT_IQ2S>(a, stream);
    case QG_FMT_IQ3S: return launch_gemv_fmt<QG_FMT_IQ3S>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qg
