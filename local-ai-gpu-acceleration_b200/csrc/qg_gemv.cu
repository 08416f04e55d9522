// qg_gemv.cu -- batch-1 quantized GEMV for sm_100a (the decode hot path).
//
// Production kernel (gemv_tiled_kernel<FMT>), one instantiation per pack format:
//  * Persistent CTAs, grid = min(tiles, SMs x resident CTAs).  A tile is a run of
//    rpp x P consecutive rows, whose payload (and Q4_K split metadata) bytes are
//    contiguous in the pack.  A dedicated producer warp streams the tile, a stage of
//    rpp x Q rows at a time, into a ring of S shared-memory stages with 1-D TMA
//    (cp.async.bulk, mbarrier completion, L2 evict-first); consumer warps release a
//    stage with one mbarrier arrive per warp, so the pipeline never needs a CTA
//    barrier.
//  * Consumer thread (slot, c) owns the 64-column chunk c: its x values are loaded
//    once, as two int8 planes, and every row's chunk is a string of dp4a
//    instructions (qg_formats.cuh).  Stages hold four passes where the shape allows
//    (fewer for matrices of two or three passes), so a thread has four independent
//    rows per stage wait.  Row sums: with full-warp lane groups (cols/64 a multiple
//    of 32) four (or two) rows at a time with one transposed butterfly, otherwise a
//    shuffle reduction in lane groups of gcd(cols/64, 32); shared-memory partials,
//    one consumer barrier per tile, then the epilogue (y, optional residual, the
//    reference's KV page word, optional peer stores of the tensor-parallel exchange).
//  * Tile size (passes per tile) chosen per shape so the tiles spread evenly over the
//    SMs (balanced_passes), capped by the shared memory left after stages and tables.
//  * IQ formats (issue- and shared-memory-bound, not HBM-bound): 16 consumer warps,
//    one CTA per SM, codebooks replicated in shared memory so that table lookups
//    spread over the banks; IQ2_S sign masks computed in registers (qg_formats.cuh).
//  * Every mbarrier wait is bounded (QG_ERR_WAIT_TIMEOUT); the producer waits for its
//    copies in flight before it exits.
//  * Two builds per format: 544 threads (96 registers per thread) and, for K-quant plans
//    of at most 480 threads at one CTA per SM, 480 threads (128 registers: the K-quant
//    readers spill at 96).
// gemv_staged_kernel<FMT> handles packs whose base address is not 16-B aligned
// (all threads copy each tile); gemv_rowwise_kernel<FMT> decodes value by value for
// rows wider than 32768 columns.
#include <algorithm>
#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>
#include <set>
#include <utility>

#include "iq_grids.h"
#include "qg_formats.cuh"
#include "qg_host.h"

namespace qg {

__device__ unsigned int g_error_word = 0u;
__device__ uint16_t g_iq2s_kgrid[1024] = {QG_IQ2S_KGRID_VALUES};
__device__ uint32_t g_iq3s_grid[512] = {QG_IQ3S_GRID_VALUES};
__device__ const ReplicatedTables g_iq2s_tables = tables_detail::make_iq2s();
__device__ const ReplicatedTables g_iq3s_tables = tables_detail::make_iq3s();

// One weight matrix of a multi-matrix launch (same format and cols): its tiles are
// [tile_end of the previous segment, tile_end).
struct GemvSeg {
  const uint8_t* payload;
  const uint8_t* meta;
  float* y;
  uint32_t rows;
  uint32_t tile_end;
};
constexpr int kMaxSegs = 3;

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
  uint32_t stage_rows;    // rows per pipeline stage (tiled kernel)
  uint32_t stage_mask;    // passes per stage - 1 (a power of two)
  uint32_t stage_shift;   // log2(passes per stage)
  uint32_t x_vec;         // x is 16-B aligned (vector loads)
  const ActChunk* xq;     // prepared activation (qg_act_prepare), or null: quantize x here
  GemvSeg seg[kMaxSegs];  // tiled kernel: the matrices of this launch (seg[0] = payload/meta/y)
  uint32_t nseg;
  uint32_t red;           // tiled kernel: passes reduced 4 or 2 at a time (group 32, Q % red == 0), else 0
  GemvExchange ex;        // tiled kernel: optional tensor-parallel exchange of the rows
  uint32_t canon_spg;     // canonical row sum: reduction groups per segment (0: plain order)
  uint32_t canon_nseg;    // canonical row sum: segments per row (1, 2, 4 or 8)
};

// Segment of tile `tile` and the tile's first row inside that segment.
__device__ __forceinline__ uint32_t tile_segment(const GemvArgs& a, uint32_t tile,
                                                 uint32_t& row0) {
  uint32_t s = 0, begin = 0;
  while (s + 1u < a.nseg && tile >= a.seg[s].tile_end) {
    begin = a.seg[s].tile_end;
    ++s;
  }
  row0 = (tile - begin) * a.rows_per_tile;
  return s;
}

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
__global__ void __launch_bounds__(512, 1) gemv_staged_kernel(const GemvArgs a) {
  constexpr uint32_t PB = FmtTraits<FMT>::payload_bytes;
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  float* red = reinterpret_cast<float*>(smem + a.red_off);
  uint8_t* stages = smem + a.stage_off;

  const uint32_t tid = threadIdx.x;
  const uint32_t nthreads = blockDim.x;
  pdl_wait();
  pdl_trigger();
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
  build_iq_tables<FMT>(smem + a.table_off, tid, nthreads);
  const IqTables tables = iq_tables<FMT>(smem + a.table_off, tid & 31u);
  XChunk xr;
  if (a.xq != nullptr) {
    load_act_chunk(a.xq + c, xr);
  } else {
    load_x_chunk(a.x + 64u * c, a.x_vec != 0u, xr);
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
        part = chunk_dot<FMT>(rp, rm, c, xr, tables);
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
  pdl_wait();
  pdl_trigger();
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
// Tiled kernel: the production path for 16-B aligned packs.

// Issue the TMA for stage `s` holding rows [row_begin, row_begin + stage_rows) of the
// pack, fewer at the end of the tile (row_end: a tile may end inside a stage) or of the
// pack.  A stage may end off a 16-B boundary: its tail bytes are copied here, before the
// arrive that publishes the stage.
template <int FMT>
__device__ __forceinline__ void tiled_issue(const GemvArgs& a, const GemvSeg& g, uint8_t* st,
                                            uint64_t* bar, uint32_t row_begin, uint32_t row_end,
                                            uint64_t policy) {
  constexpr uint32_t PB = FmtTraits<FMT>::payload_bytes;
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  const uint32_t bpr = a.cols >> 8;
  const uint32_t limit = min(g.rows, row_end);
  uint32_t nr = 0u;
  if (row_begin < limit) nr = min(a.stage_rows, limit - row_begin);
  const uint32_t pb = nr * bpr * PB, mb = nr * bpr * MB;
  const uint32_t pb16 = pb & ~15u, mb16 = mb & ~15u;
  const uint8_t* src = g.payload + static_cast<uint64_t>(row_begin) * bpr * PB;
  const uint8_t* msrc = g.meta + static_cast<uint64_t>(row_begin) * bpr * MB;
  for (uint32_t o = pb16; o < pb; ++o) st[o] = src[o];
  if (MB != 0u) {
    for (uint32_t o = mb16; o < mb; ++o) st[a.meta_off + o] = msrc[o];
  }
  mbar_arrive_expect_tx(bar, pb16 + mb16);
  if (pb16 != 0u) tma_load_1d(st, src, pb16, bar, policy);
  if (MB != 0u && mb16 != 0u) tma_load_1d(st + a.meta_off, msrc, mb16, bar, policy);
}

__device__ __forceinline__ void consumer_sync(uint32_t nconsumers) {
  asm volatile("bar.sync 1, %0;" ::"r"(nconsumers) : "memory");
}

// Sum over an aligned lane group of `group` lanes (4, 8, 16 or 32; warp-uniform).
__device__ __forceinline__ float group_sum(float v, uint32_t group) {
  if (group > 16u) v += __shfl_xor_sync(0xffffffffu, v, 16);
  if (group > 8u) v += __shfl_xor_sync(0xffffffffu, v, 8);
  if (group > 4u) v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v;
}

// Sums four per-lane values over each aligned group of G lanes (G = 4, 8, 16 or 32,
// warp-uniform) at once, a transposed butterfly: the first two exchanges (lane bits G/2
// and G/4) trade one value of a pair instead of both (for G = 32: 6 shuffles for four
// sums instead of 20).  Lane l ends with the total of v[2 * bit(G/4) + bit(G/2)], so the
// lanes whose bits below G/4 are zero hold the group's four sums.  Every sum is the
// same tree as group_sum's: pairs differing in lane bit G/2 first, then G/4, ..., 1.
__device__ __forceinline__ float warp_sum4(const float (&v)[4], uint32_t lane, uint32_t G) {
  const uint32_t h = G >> 1, q = G >> 2;
  const bool bh = (lane & h) != 0u, bq = (lane & q) != 0u;
  const float w0 = (bh ? v[1] : v[0]) + __shfl_xor_sync(0xffffffffu, bh ? v[0] : v[1], h);
  const float w1 = (bh ? v[3] : v[2]) + __shfl_xor_sync(0xffffffffu, bh ? v[2] : v[3], h);
  float u = (bq ? w1 : w0) + __shfl_xor_sync(0xffffffffu, bq ? w0 : w1, q);
  for (uint32_t off = G >> 3; off > 0u; off >>= 1) u += __shfl_xor_sync(0xffffffffu, u, off);
  return u;
}

// The two-value form: lane l ends with the total of v[bit(G/2)] (the lanes whose bits
// below G/2 are zero hold the group's two sums).
__device__ __forceinline__ float warp_sum2(const float (&v)[2], uint32_t lane, uint32_t G) {
  const uint32_t h = G >> 1;
  const bool bh = (lane & h) != 0u;
  float u = (bh ? v[1] : v[0]) + __shfl_xor_sync(0xffffffffu, bh ? v[0] : v[1], h);
  for (uint32_t off = G >> 2; off > 0u; off >>= 1) u += __shfl_xor_sync(0xffffffffu, u, off);
  return u;
}

// Row total from the row's group partials p[0..gpr) in the canonical order (tensor-
// parallel row-parallel matrices; the plain order is p[0] + p[1] + ...): the row is `nseg` segments of
// `spg` consecutive groups; each segment is summed left to right, then the segments in
// a pairwise tree.  A segment is one tensor-parallel shard at the largest TP degree, so
// a rank holding a power-of-two run of segments computes a complete subtree, and the
// exchange that adds the ranks' results in the same pairwise tree (gather kernel)
// reproduces the single-GPU sum bit for bit.
__device__ __forceinline__ float row_total(const float* p, uint32_t gpr, uint32_t spg,
                                        uint32_t nseg) {
  (void)gpr;
  float seg[8];
#pragma unroll
  for (uint32_t s = 0; s < 8u; ++s) {
    if (s < nseg) {
      float acc = p[s * spg];
      for (uint32_t k = 1; k < spg; ++k) acc += p[s * spg + k];
      seg[s] = acc;
    }
  }
#pragma unroll
  for (uint32_t step = 1; step < 8u; step <<= 1) {
#pragma unroll
    for (uint32_t i = 0; i + step < 8u; i += 2u * step) {
      if (i + step < nseg) seg[i] += seg[i + step];
    }
  }
  return seg[0];
}

// CANON: row sums in the canonical segment order (row_total) with lane groups of
// a.group chunks; otherwise lane groups of 32 chunks reduce with the transposed
// butterflies (red = 4 or 2) and narrower groups with group_sum.
template <int FMT, bool CANON, uint32_t MAXT>
__global__ void __launch_bounds__(MAXT, 1) gemv_tiled_kernel(const GemvArgs a) {
  constexpr uint32_t PB = FmtTraits<FMT>::payload_bytes;
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + 8;
  float* red = reinterpret_cast<float*>(smem + a.red_off);
  uint8_t* stages = smem + a.stage_off;

  const uint32_t tid = threadIdx.x, lane = tid & 31u;
  const uint32_t nconsumers = blockDim.x - 32u;  // the last warp is the producer
  const uint32_t first = blockIdx.x, stride = gridDim.x;
  const uint32_t n_my = a.num_tiles > first ? (a.num_tiles - first + stride - 1u) / stride : 0u;
  // a tile is passes rows-passes; its last stage may be partial
  const uint32_t loads_per_tile = (a.passes + a.stage_mask) >> a.stage_shift;
  const uint32_t S = a.stages;

  uint64_t* table_bar = full + 16;
  constexpr bool kTables = FMT == QG_FMT_IQ2S || FMT == QG_FMT_IQ3S;
  if (tid == 0u) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&full[s], 1u);
      mbar_init(&empty[s], nconsumers >> 5);
    }
    mbar_init(table_bar, 1u);
    fence_mbar_init();
  }
  __syncthreads();

  if (tid >= nconsumers) {
    // Producer warp: one elected lane streams every stage of this CTA's tiles.
    if (lane == 0u) {
      const uint64_t policy = l2_evict_first_policy();
      if (kTables) {
        // The codebook tables (64 KB, L2-resident after the first CTA) in one bulk copy.
        mbar_arrive_expect_tx(table_bar, iq_table_bytes(FMT));
        tma_load_1d(smem + a.table_off, replicated_tables<FMT>(), iq_table_bytes(FMT),
                    table_bar);
      }
      bool ok = true;
      uint32_t s = 0, ephase = 0, issued = 0;
      for (uint32_t i = 0; i < n_my && ok; ++i) {
        uint32_t row0;
        const GemvSeg& g = a.seg[tile_segment(a, first + i * stride, row0)];
        for (uint32_t j = 0; j < loads_per_tile; ++j) {
          if (issued >= S) {
            ok = mbar_wait_bounded(&empty[s], ephase);
            if (!ok) break;
          }
          tiled_issue<FMT>(a, g, stages + s * a.stage_bytes, &full[s], row0 + j * a.stage_rows,
                           row0 + a.rows_per_tile, policy);
          ++issued;
          if (++s == S) {
            s = 0;
            if (issued > S) ephase ^= 1u;
          }
        }
      }
      // Copies still in flight must land before this CTA's shared memory is released:
      // wait for the last min(S, issued) stages (bounded).
      if (ok) {
        const uint32_t n = min(S, issued);
        for (uint32_t k = 0; k < n; ++k) {
          const uint32_t L = issued - n + k;
          mbar_wait_bounded(&full[L % S], (L / S) & 1u);
        }
      }
    }
    return;
  }

  const bool valid = tid < a.rpp * a.tpr;
  const uint32_t slot = valid ? tid / a.tpr : 0u;
  const uint32_t c = valid ? tid - slot * a.tpr : 0u;
  const uint32_t bpr = a.cols >> 8;
  const uint32_t gpr = a.tpr / a.group;
  const uint32_t gidx = c / a.group;
  const bool leader = valid && (c & (a.group - 1u)) == 0u;
  const uint32_t row_stride = bpr * PB, meta_stride = bpr * MB;
  const uint32_t Q = a.stage_rows / a.rpp;
  const uint32_t G = CANON ? a.group : 32u;

  const IqTables tables = iq_tables<FMT>(smem + a.table_off, tid & 31u);
  pdl_wait();  // x / act / residual / token come from the previous kernel
  pdl_trigger();
  XChunk xr;
  if (a.xq != nullptr) {
    load_act_chunk(a.xq + c, xr);
  } else {
    load_x_chunk(a.x + 64u * c, a.x_vec != 0u, xr);
  }
  const uint32_t tok = (a.kv != nullptr && a.token != nullptr) ? *a.token : 0u;
  // exchange epoch of this launch and the parity half of the ranks' buffers it fills
  const uint32_t ex_epoch = a.ex.n != 0u ? *a.ex.epoch + 1u : 0u;
  const uint32_t ex_off = (ex_epoch & 1u) * a.ex.stride;
  bool failed = false;
  if (kTables && !mbar_wait_bounded(table_bar, 0u)) failed = true;

  uint32_t s = 0, phase = 0;
  for (uint32_t i = 0; i < n_my && !failed; ++i) {
    uint32_t row0;
    const GemvSeg& g = a.seg[tile_segment(a, first + i * stride, row0)];
    const uint32_t nrows = min(a.rows_per_tile, g.rows - row0);
    float* rb = red + (i & 1u) * (a.rows_per_tile * gpr);
    for (uint32_t j = 0; j < loads_per_tile; ++j) {
      if (!mbar_wait_bounded(&full[s], phase)) failed = true;
      const uint8_t* st = stages + s * a.stage_bytes;
      const uint32_t lr0 = j * a.stage_rows + slot;  // tile row of q = 0
      if (a.red == 4u) {
        // Each lane group covers G chunks of one row slot: four passes' chunks, then one
        // transposed reduction for the four rows.
        for (uint32_t q = 0; q < Q; q += 4u) {
          float v[4];
#pragma unroll
          for (uint32_t r = 0; r < 4u; ++r) {
            // Decoded unconditionally and selected, so the rows form one block the
            // compiler can interleave: a row past the tile (or a thread past the pass)
            // reads stale bytes of this stage -- inside the stage buffer, every codebook
            // index in range -- and its value is dropped.
            const uint32_t lr = lr0 + (q + r) * a.rpp;
            const uint32_t ls = (q + r) * a.rpp + slot;
            const float val = chunk_dot<FMT>(st + ls * row_stride, st + a.meta_off + ls * meta_stride,
                                             c, xr, tables);
            v[r] = (valid && lr < nrows && !failed) ? val : 0.f;
          }
          const float u = warp_sum4(v, lane, G);
          const uint32_t lr = lr0 + (q + ((lane & (G >> 2)) ? 2u : 0u) + ((lane & (G >> 1)) ? 1u : 0u)) * a.rpp;
          if ((lane & ((G >> 2) - 1u)) == 0u && valid && lr < nrows && !failed) rb[lr * gpr + gidx] = u;
        }
      } else if (a.red == 2u) {
        for (uint32_t q = 0; q < Q; q += 2u) {
          float v[2];
#pragma unroll
          for (uint32_t r = 0; r < 2u; ++r) {
            // Decoded unconditionally and selected, so the rows form one block the
            // compiler can interleave: a row past the tile (or a thread past the pass)
            // reads stale bytes of this stage -- inside the stage buffer, every codebook
            // index in range -- and its value is dropped.
            const uint32_t lr = lr0 + (q + r) * a.rpp;
            const uint32_t ls = (q + r) * a.rpp + slot;
            const float val = chunk_dot<FMT>(st + ls * row_stride, st + a.meta_off + ls * meta_stride,
                                             c, xr, tables);
            v[r] = (valid && lr < nrows && !failed) ? val : 0.f;
          }
          const float u = warp_sum2(v, lane, G);
          const uint32_t lr = lr0 + (q + ((lane & (G >> 1)) ? 1u : 0u)) * a.rpp;
          if ((lane & ((G >> 1) - 1u)) == 0u && valid && lr < nrows && !failed) rb[lr * gpr + gidx] = u;
        }
      }
#pragma unroll 2
      for (uint32_t q = 0; a.red == 0u && q < Q; ++q) {
        const uint32_t lr = lr0 + q * a.rpp;
        const bool live = valid && lr < nrows && !failed;
        float part = 0.f;
        if (live) {
          const uint32_t ls = q * a.rpp + slot;
          part = chunk_dot<FMT>(st + ls * row_stride, st + a.meta_off + ls * meta_stride, c, xr,
                                tables);
        }
        part = group_sum(part, a.group);
        if (leader && live) rb[lr * gpr + gidx] = part;
      }
      __syncwarp();
      if (lane == 0u) mbar_arrive(&empty[s]);
      if (++s == S) {
        s = 0;
        phase ^= 1u;
      }
    }
    consumer_sync(nconsumers);
    for (uint32_t t = tid; t < nrows; t += nconsumers) {
      float v;
      if constexpr (CANON) {
        v = row_total(rb + t * gpr, gpr, a.canon_spg, a.canon_nseg);
      } else {
        v = 0.f;
        for (uint32_t k = 0; k < gpr; ++k) v += rb[t * gpr + k];
      }
      const uint32_t row = row0 + t;
      if (a.residual != nullptr) v = a.residual[row] + v;
      g.y[row] = v;
      if (a.ex.n != 0u) {  // NVLink peer stores of (epoch, value)
        const uint64_t word = (static_cast<uint64_t>(ex_epoch) << 32) | __float_as_uint(v);
        for (uint32_t p = 0; p < a.ex.n; ++p) st_relaxed_sys_u64(a.ex.out[p] + ex_off + row, word);
      }
      if (a.kv != nullptr && row < a.active_pages && a.kv_words > 0u && a.page_words > 0u) {
        const uint64_t kb = static_cast<uint64_t>(row) * a.page_words;
        const uint64_t ko = (tok + row) % a.page_words;
        a.kv[(kb + ko) % a.kv_words] = v;
      }
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

template <typename K>
cudaError_t ensure_smem_attr(K kernel, int max_optin) {
  // One attribute set per (kernel, device); cudaFuncSetAttribute is cheap but not free.
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key) == 0u) {
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_optin);
    if (e != cudaSuccess) return e;
    done.insert(key);
  }
  return cudaSuccess;
}

// Resident CTAs per SM for a kernel at a block size and dynamic smem (cached).
template <typename K>
uint32_t resident_ctas(K kernel, uint32_t threads, uint32_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, uint32_t, uint32_t, int>, uint32_t> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(reinterpret_cast<const void*>(kernel), threads, smem, dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, static_cast<int>(threads), smem) !=
          cudaSuccess ||
      n < 1) {
    n = 1;
  }
  cache[key] = static_cast<uint32_t>(n);
  return static_cast<uint32_t>(n);
}

uint32_t ctas_per_sm(const GemvPlan& p);

// The build of the tiled kernel for a plan.  Registers are allocated per SM
// sub-partition (16384 each), so the 17-warp build (544 threads) leaves 96 per thread, at
// which the K-quant readers spill; K-quant plans of at most 480 threads that run one CTA
// per SM take the 15-warp build (128 registers per thread).  IQ plans always use 544.
template <int FMT, bool CANON>
void (*tiled_kernel_for(const GemvPlan& plan))(const GemvArgs) {
  if constexpr (iq_table_bytes(FMT) == 0u) {
    if (plan.threads <= 480u && ctas_per_sm(plan) == 1u) return gemv_tiled_kernel<FMT, CANON, 480u>;
  }
  return gemv_tiled_kernel<FMT, CANON, 544u>;
}

void fill_args(GemvArgs& a, const GemvPlan& plan, bool canon = false) {
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
  a.stage_rows = plan.stage_rows;
  a.stage_mask = plan.stage_passes - 1u;
  a.stage_shift = static_cast<uint32_t>(__builtin_ctz(plan.stage_passes));
  a.red = 0u;
  if (plan.tiled != 0u && (plan.group == 32u || (canon && plan.group >= 4u))) {
    a.red = (plan.stage_passes & 3u) == 0u ? 4u : (plan.stage_passes & 1u) == 0u ? 2u : 0u;
  }
}

template <int FMT>
cudaError_t launch_gemv_fmt(GemvArgs a, cudaStream_t stream) {
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  const DeviceInfo dev = device_info();
  a.tpr = a.cols / 64u;
  a.x_vec = (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0u ? 1u : 0u;
  if (a.cols < 256u || a.tpr > 512u) {
    return launch_k(gemv_rowwise_kernel<FMT>, a.rows, 256, 0, stream, a);
  }
  const bool aligned = (reinterpret_cast<uintptr_t>(a.payload) & 15u) == 0u &&
                       (MB == 0u || (reinterpret_cast<uintptr_t>(a.meta) & 15u) == 0u);
  if (aligned) {
    const GemvPlan plan = plan_gemv(FMT, a.rows, a.cols, dev.sms);
    if (plan.tiled && plan.smem_bytes <= static_cast<uint32_t>(dev.max_smem_optin)) {
      fill_args(a, plan);
      a.tma_ok = 1u;
      a.nseg = 1u;
      a.seg[0] = GemvSeg{a.payload, a.meta, a.y, a.rows, plan.num_tiles};
      const auto kernel = tiled_kernel_for<FMT, false>(plan);
      const cudaError_t e = ensure_smem_attr(kernel, dev.max_smem_optin);
      if (e != cudaSuccess) return e;
      const uint32_t per_sm = resident_ctas(kernel, plan.threads, plan.smem_bytes);
      const uint32_t grid = std::max(1u, std::min(plan.num_tiles, per_sm * dev.sms));
      return launch_k(kernel, grid, plan.threads, plan.smem_bytes, stream, a);
    }
  }
  // Unaligned packs (or shapes the tiled plan cannot stage): all-thread copies.
  const GemvPlan plan = plan_staged(FMT, a.rows, a.cols, dev.sms);
  if (plan.smem_bytes > static_cast<uint32_t>(dev.max_smem_optin)) {
    return launch_k(gemv_rowwise_kernel<FMT>, a.rows, 256, 0, stream, a);
  }
  fill_args(a, plan);
  a.tma_ok = 0u;
  const cudaError_t e = ensure_smem_attr(gemv_staged_kernel<FMT>, dev.max_smem_optin);
  if (e != cudaSuccess) return e;
  const uint32_t per_sm = resident_ctas(gemv_staged_kernel<FMT>, plan.threads, plan.smem_bytes);
  const uint32_t grid = std::max(1u, std::min(plan.num_tiles, per_sm * dev.sms));
  return launch_k(gemv_staged_kernel<FMT>, grid, plan.threads, plan.smem_bytes, stream, a);
}

// Several matrices of one format and width that read the same x, in one launch (the
// Q/K/V projections, gate/up).  Falls back to one launch per matrix when a matrix is
// not 16-B aligned or the shape cannot use the tiled kernel.
template <int FMT>
cudaError_t launch_multi_fmt(GemvArgs a, uint32_t nseg, const GemvSeg* segs, cudaStream_t stream) {
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  const DeviceInfo dev = device_info();
  a.tpr = a.cols / 64u;
  a.x_vec = (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0u ? 1u : 0u;
  bool aligned = a.cols >= 256u && a.tpr <= 512u;
  uint32_t total_rows = 0;
  for (uint32_t k = 0; k < nseg; ++k) {
    aligned = aligned && (reinterpret_cast<uintptr_t>(segs[k].payload) & 15u) == 0u &&
              (MB == 0u || (reinterpret_cast<uintptr_t>(segs[k].meta) & 15u) == 0u);
    total_rows += segs[k].rows;
  }
  GemvPlan plan{};
  if (aligned) plan = plan_gemv(FMT, total_rows, a.cols, dev.sms);
  if (!aligned || !plan.tiled || plan.smem_bytes > static_cast<uint32_t>(dev.max_smem_optin)) {
    for (uint32_t k = 0; k < nseg; ++k) {
      GemvArgs b = a;
      b.payload = segs[k].payload;
      b.meta = segs[k].meta;
      b.y = segs[k].y;
      b.rows = segs[k].rows;
      const cudaError_t e = launch_gemv_fmt<FMT>(b, stream);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  fill_args(a, plan);
  a.tma_ok = 1u;
  a.nseg = nseg;
  uint32_t tiles = 0;
  for (uint32_t k = 0; k < nseg; ++k) {
    a.seg[k] = segs[k];
    tiles += (segs[k].rows + plan.rows_per_tile - 1u) / plan.rows_per_tile;
    a.seg[k].tile_end = tiles;
  }
  a.num_tiles = tiles;
  a.payload = segs[0].payload;
  a.meta = segs[0].meta;
  a.y = segs[0].y;
  a.rows = segs[0].rows;
  const auto kernel = tiled_kernel_for<FMT, false>(plan);
  const cudaError_t e = ensure_smem_attr(kernel, dev.max_smem_optin);
  if (e != cudaSuccess) return e;
  const uint32_t per_sm = resident_ctas(kernel, plan.threads, plan.smem_bytes);
  const uint32_t grid = std::max(1u, std::min(tiles, per_sm * dev.sms));
  return launch_k(kernel, grid, plan.threads, plan.smem_bytes, stream, a);
}

// Threads per CTA: rows-per-pass is the smallest multiple of 32/group (whole warps)
// that reaches ~256 threads; rows wider than 512 threads pad the last warp.
#ifndef QG_IQ_THREADS
#define QG_IQ_THREADS 512u
#endif
#ifndef QG_IQ_STAGE_PASSES
#define QG_IQ_STAGE_PASSES 4u
#endif
#ifndef QG_STAGE_PASSES
#define QG_STAGE_PASSES 4u
#endif
#ifndef QG_THREADS
#define QG_THREADS 256u
#endif
#ifndef QG_IQ_STAGE_BUDGET
#define QG_IQ_STAGE_BUDGET (96u * 1024u)
#endif
constexpr uint32_t kIqThreads = QG_IQ_THREADS;
constexpr uint32_t kIqStagePasses = QG_IQ_STAGE_PASSES;
constexpr uint32_t kStagePasses = QG_STAGE_PASSES;
constexpr uint32_t kThreads = QG_THREADS;
// Dynamic shared memory a CTA may opt into on sm_100 (227 KB).
constexpr uint32_t kSmemOptinMax = 232448u;
constexpr uint32_t kIqStageBudget = QG_IQ_STAGE_BUDGET;

void plan_threads(uint32_t tpr, GemvPlan& p, uint32_t limit = 256u, uint32_t group_cap = 32u) {
  p.group = gcd_u32(tpr, group_cap);
  const uint32_t base = 32u / p.group;
  uint32_t rpp = base;
  if (rpp * tpr > 512u) rpp = 1u;
  while ((rpp + base) * tpr <= limit) rpp += base;
  p.rpp = rpp;
  p.threads = ((rpp * tpr + 31u) / 32u) * 32u;
}

void plan_smem(int fmt, uint32_t tpr, GemvPlan& p) {
  const uint32_t red_floats = 2u * p.rows_per_tile * (tpr / p.group);
  p.red_off = 256u;  // 16 mbarriers
  p.table_off = (p.red_off + red_floats * 4u + 127u) & ~127u;
  const uint32_t table_bytes = iq_table_bytes(fmt);
  p.stage_off = (p.table_off + table_bytes + 127u) & ~127u;
  p.smem_bytes = p.stage_off + p.stages * p.stage_bytes;
}

// Resident CTAs per SM of a plan (the tiled kernels are built for <= 96 registers).
uint32_t ctas_per_sm(const GemvPlan& p) {
  const uint32_t by_smem = std::max(1u, (228u * 1024u) / (p.smem_bytes + 1024u));
  const uint32_t by_threads = std::max(1u, 2048u / p.threads);
  const uint32_t by_regs = std::max(1u, 65536u / (((p.threads + 31u) / 32u) * 32u * 96u));
  return std::min(by_smem, std::min(by_threads, by_regs));
}

// Passes per tile.  Tiles go round-robin to the G = min(T, slots) persistent CTAs, so
// CTA j runs ceil(T / G) or one fewer tiles, and an SM runs whichever m CTAs the block
// scheduler put on it (m = CTAs per SM when G exceeds the SM count, else 1).  Cost of
// a tile size P (a multiple of the stage's q passes, or of q_align, the fewest passes
// whose bytes are 16-B aligned, when a tile may end inside a stage; at most p_max): the
// tiles of the m busiest CTAs times (P + 1/2) -- the half pass stands for a tile's
// barrier and epilogue -- divided by 0.6 when a CTA sized to share its SM runs alone
// (measured on B200: one 9-warp CTA streams ~0.6 of what two do).  Ties go to the
// larger P.
double tile_cost(uint32_t total_passes, uint32_t P, uint32_t sms, uint32_t cps) {
  const uint32_t slots = sms * cps;
  const uint32_t T = (total_passes + P - 1u) / P;
  const uint32_t G = std::min(T, slots);
  const uint32_t k = (T + G - 1u) / G;         // tiles of the busiest CTAs
  const uint32_t n_k = T - (k - 1u) * G;        // CTAs with k tiles
  const uint32_t m = G > sms ? cps : 1u;        // CTAs sharing the busiest SM
  const uint32_t tiles = n_k >= m ? m * k : n_k * k + (m - n_k) * (k - 1u);
  double cost = static_cast<double>(tiles) * (2.0 * P + 1.0);
  if (cps > 1u && G <= sms) cost /= 0.6;
  return cost;
}

// Best P in steps of `step` (ties to the larger P).
uint32_t best_passes(uint32_t total_passes, uint32_t step, uint32_t sms, uint32_t cps,
                     uint32_t p_max, double& best_cost) {
  uint32_t best_p = step;
  best_cost = 1e300;
  for (uint32_t P = step; P <= std::max(step, p_max); P += step) {
    const double cost = tile_cost(total_passes, P, sms, cps);
    if (cost <= best_cost) {
      best_cost = cost;
      best_p = P;
    }
  }
  return best_p;
}

// Tiles are whole stages (q passes) unless tiles that end inside a stage (multiples of
// q_align) balance at least 2% better -- the medium matrices whose rows do not spread
// over the SMs in whole stages (e.g. 10240 x 8192: 20-pass tiles on 128 CTAs against
// 18-pass tiles on 143).
uint32_t balanced_passes(uint32_t total_passes, uint32_t q, uint32_t q_align, uint32_t sms,
                         uint32_t cps, uint32_t p_max) {
  double whole = 0.0, fine = 0.0;
  const uint32_t pw = best_passes(total_passes, q, sms, cps, std::max(q, p_max - p_max % q), whole);
  const uint32_t pf = best_passes(total_passes, q_align, sms, cps,
                                  std::max(q_align, p_max - p_max % q_align), fine);
  return fine < 0.98 * whole ? pf : pw;
}

}  // namespace

// Plan of the tiled kernel.  Stage = Q passes of ~16 KB whose byte count is a multiple
// of 16 (IQ formats: at least four passes); S stages within ~96 KB (2..8); tiles of P
// passes balanced over the SMs (balanced_passes: whole stages, or ending inside one when
// that balances better).
GemvPlan plan_gemv(int fmt, uint32_t rows, uint32_t cols, int sms, uint32_t group_cap) {
  GemvPlan p{};
  sms = std::max(sms, 1);  // no device (host-side plan query): plan for one SM
  const uint32_t PB = qg_payload_bytes_per_block(fmt);
  const uint32_t MB = qg_meta_bytes_per_block(fmt);
  const uint32_t bpr = cols >> 8, tpr = cols / 64u;
  const bool iq = iq_table_bytes(fmt) != 0u;
  plan_threads(tpr, p, iq ? kIqThreads : kThreads, group_cap);
  const uint32_t row_bytes = bpr * PB, row_meta = bpr * MB;
  // Stage: smallest power-of-two passes with 16-B aligned bytes, grown toward 16 KB.
  uint32_t q = 1u;
  while (q <= 32u && (((q * p.rpp * row_bytes) & 15u) != 0u || ((q * p.rpp * row_meta) & 15u) != 0u)) {
    q <<= 1;
  }
  if (q > 32u) {
    p.tiled = 0u;
    return p;
  }
  const uint32_t q_align = q;
  const uint32_t stage_target = iq ? 8192u : 16384u;
  while (q < 16u && 2u * q * p.rpp * (row_bytes + row_meta) <= stage_target) q <<= 1;
  // IQ readers are issue-bound: four passes per stage give every thread four
  // independent chunks and one transposed reduction per four rows.
  // (Canonical-order plans, group_cap < 32, keep the same four passes.)
  if (p.group == 32u || group_cap < 32u) q = std::max(q, iq ? kIqStagePasses : kStagePasses);
  const uint32_t total_passes = std::max(1u, (rows + p.rpp - 1u) / p.rpp);
  // Small matrices: a stage is never more passes than the matrix has (but never less
  // than its 16-B aligned size).
  while (q > q_align && q > total_passes) q >>= 1;
  // Two stages of q passes, the codebooks and the reduction buffer of tiles of at least
  // 16 passes must fit the 227 KB a CTA may opt into (else the launch would drop to the
  // all-thread kernels); the tile size is then capped by what is left.
  const uint32_t red_per_pass = 2u * p.rpp * (tpr / p.group) * 4u;  // double-buffered floats
  auto stage_of = [&](uint32_t qq) {
    return ((qq * p.rpp * row_bytes + 127u) & ~127u) + ((qq * p.rpp * row_meta + 127u) & ~127u);
  };
  auto fixed_of = [&](uint32_t qq) { return 2u * stage_of(qq) + iq_table_bytes(fmt) + 1024u; };
  while (q > q_align && fixed_of(q) + 16u * red_per_pass > kSmemOptinMax) q >>= 1;
  const uint32_t p_max =
      fixed_of(q) < kSmemOptinMax ? std::min(128u, (kSmemOptinMax - fixed_of(q)) / red_per_pass) : q;
  p.stage_passes = q;
  p.stage_rows = q * p.rpp;
  const uint32_t pay = p.stage_rows * row_bytes, met = p.stage_rows * row_meta;
  p.meta_off = (pay + 127u) & ~127u;
  p.stage_bytes = MB ? ((p.meta_off + met + 127u) & ~127u) : ((pay + 127u) & ~127u);
  const uint32_t budget = iq ? kIqStageBudget : 96u * 1024u;
  p.stages = std::max(2u, std::min(8u, budget / p.stage_bytes));
  p.threads += 32u;  // producer warp
  // Resident CTAs per SM from the smallest tile, then the balanced tile size.
  p.passes = q;
  p.rows_per_tile = q * p.rpp;
  plan_smem(fmt, tpr, p);
  const uint32_t cps = ctas_per_sm(p);
  const uint32_t P = balanced_passes(total_passes, q, q_align, static_cast<uint32_t>(sms), cps,
                                     std::max(q, p_max));
  p.passes = P;
  p.rows_per_tile = P * p.rpp;
  p.num_tiles = (rows + p.rows_per_tile - 1u) / p.rows_per_tile;
  plan_smem(fmt, tpr, p);
  p.grid = std::max(1u, std::min(p.num_tiles, static_cast<uint32_t>(sms) * ctas_per_sm(p)));
  p.tiled = 1u;
  return p;
}

// Plan of the all-thread-copy kernel (one row pass per thread per tile row group).
GemvPlan plan_staged(int fmt, uint32_t rows, uint32_t cols, int sms) {
  GemvPlan p{};
  const uint32_t PB = qg_payload_bytes_per_block(fmt);
  const uint32_t MB = qg_meta_bytes_per_block(fmt);
  const uint32_t bpr = cols >> 8, tpr = cols / 64u;
  plan_threads(tpr, p);
  const uint32_t row_bytes = bpr * PB, row_meta = bpr * MB;
  const uint32_t passes = std::max(1u, std::min(4u, 16384u / std::max(1u, p.rpp * row_bytes)));
  p.passes = passes;
  p.stage_passes = 1u;
  p.rows_per_tile = passes * p.rpp;
  p.stage_rows = p.rows_per_tile;
  p.num_tiles = (rows + p.rows_per_tile - 1u) / p.rows_per_tile;
  const uint32_t pay = p.rows_per_tile * row_bytes, met = p.rows_per_tile * row_meta;
  p.meta_off = (pay + 127u) & ~127u;
  p.stage_bytes = MB ? ((p.meta_off + met + 127u) & ~127u) : ((pay + 127u) & ~127u);
  p.stages = std::max(2u, std::min(8u, (96u * 1024u) / p.stage_bytes));
  plan_smem(fmt, tpr, p);
  p.grid = std::max(1u, std::min(p.num_tiles, static_cast<uint32_t>(sms) * ctas_per_sm(p)));
  p.tiled = 0u;
  return p;
}

cudaError_t launch_gemv(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                        const void* act, float* y, const float* residual, float* kv,
                        const uint32_t* token, uint64_t kv_words, uint32_t page_words,
                        uint32_t active_pages, uint32_t rows, uint32_t cols, cudaStream_t stream) {
  GemvArgs a{};
  a.payload = payload;
  a.meta = meta;
  a.x = x;
  a.xq = static_cast<const ActChunk*>(act);
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

namespace {
// Tiled launch whose row sums follow the canonical segment order (canon.seg_chunks
// 64-column chunks per segment, a multiple of 4, so lane groups are at least 4 wide;
// canon.nseg segments per row), optionally exchanging the rows with the other ranks.  cudaErrorNotSupported when the shape, the alignment or
// the segment size does not allow the tiled kernel.
template <int FMT>
cudaError_t launch_canon_fmt(GemvArgs a, const GemvCanon& canon, cudaStream_t stream) {
  constexpr uint32_t MB = FmtTraits<FMT>::meta_bytes;
  const DeviceInfo dev = device_info();
  a.tpr = a.cols / 64u;
  a.x_vec = (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0u ? 1u : 0u;
  const bool aligned = (reinterpret_cast<uintptr_t>(a.payload) & 15u) == 0u &&
                       (MB == 0u || (reinterpret_cast<uintptr_t>(a.meta) & 15u) == 0u);
  if (a.cols < 256u || a.tpr > 512u || !aligned) return cudaErrorNotSupported;
  if (canon.nseg == 0u || canon.nseg > 8u || (canon.nseg & (canon.nseg - 1u)) != 0u ||
      canon.seg_chunks % 4u != 0u || canon.seg_chunks == 0u || canon.seg_chunks * canon.nseg != a.tpr) {
    return cudaErrorInvalidValue;
  }
  const uint32_t cg = gcd_u32(canon.seg_chunks, 32u);
  const GemvPlan plan = plan_gemv(FMT, a.rows, a.cols, dev.sms, cg);
  if (!plan.tiled || plan.smem_bytes > static_cast<uint32_t>(dev.max_smem_optin) || plan.group != cg) {
    return cudaErrorNotSupported;
  }
  fill_args(a, plan, true);
  a.tma_ok = 1u;
  a.nseg = 1u;
  a.seg[0] = GemvSeg{a.payload, a.meta, a.y, a.rows, plan.num_tiles};
  a.canon_spg = canon.seg_chunks / cg;
  a.canon_nseg = canon.nseg;
  const auto kernel = tiled_kernel_for<FMT, true>(plan);
  const cudaError_t e = ensure_smem_attr(kernel, dev.max_smem_optin);
  if (e != cudaSuccess) return e;
  const uint32_t per_sm = resident_ctas(kernel, plan.threads, plan.smem_bytes);
  const uint32_t grid = std::max(1u, std::min(plan.num_tiles, per_sm * dev.sms));
  return launch_k(kernel, grid, plan.threads, plan.smem_bytes, stream, a);
}

cudaError_t launch_canon(int fmt, const GemvArgs& a, const GemvCanon& canon, cudaStream_t stream) {
  switch (fmt) {
    case QG_FMT_Q4K_RAW: return launch_canon_fmt<QG_FMT_Q4K_RAW>(a, canon, stream);
    case QG_FMT_Q4K_SPLIT_PREDECODED: return launch_canon_fmt<QG_FMT_Q4K_SPLIT_PREDECODED>(a, canon, stream);
    case QG_FMT_Q4K_SPLIT_HALF: return launch_canon_fmt<QG_FMT_Q4K_SPLIT_HALF>(a, canon, stream);
    case QG_FMT_Q4K_SPLIT_COMPACT: return launch_canon_fmt<QG_FMT_Q4K_SPLIT_COMPACT>(a, canon, stream);
    case QG_FMT_Q4K_SPLIT_NATIVE: return launch_canon_fmt<QG_FMT_Q4K_SPLIT_NATIVE>(a, canon, stream);
    case QG_FMT_Q5K: return launch_canon_fmt<QG_FMT_Q5K>(a, canon, stream);
    case QG_FMT_IQ2S: return launch_canon_fmt<QG_FMT_IQ2S>(a, canon, stream);
    case QG_FMT_IQ3S: return launch_canon_fmt<QG_FMT_IQ3S>(a, canon, stream);
    default: return cudaErrorInvalidValue;
  }
}
}  // namespace

cudaError_t launch_gemv_exchange(int fmt, const uint8_t* payload, const uint8_t* meta,
                                 const float* x, const void* act, float* y, const float* residual,
                                 uint32_t rows, uint32_t cols, const GemvExchange& ex,
                                 const GemvCanon& canon, cudaStream_t stream) {
  if (ex.n == 0u || ex.n > kMaxExchangeRanks || ex.epoch == nullptr) {
    return cudaErrorInvalidValue;
  }
  GemvArgs a{};
  a.payload = payload;
  a.meta = meta;
  a.x = x;
  a.xq = static_cast<const ActChunk*>(act);
  a.y = y;
  a.residual = residual;
  a.rows = rows;
  a.cols = cols;
  a.ex = ex;
  return launch_canon(fmt, a, canon, stream);
}

cudaError_t launch_gemv_canonical(int fmt, const uint8_t* payload, const uint8_t* meta,
                                  const float* x, const void* act, float* y, const float* residual,
                                  uint32_t rows, uint32_t cols, const GemvCanon& canon,
                                  cudaStream_t stream) {
  GemvArgs a{};
  a.payload = payload;
  a.meta = meta;
  a.x = x;
  a.xq = static_cast<const ActChunk*>(act);
  a.y = y;
  a.residual = residual;
  a.rows = rows;
  a.cols = cols;
  return launch_canon(fmt, a, canon, stream);
}

cudaError_t launch_gemv_multi(int fmt, uint32_t nseg, const uint8_t* const* payload,
                              const uint8_t* const* meta, float* const* y, const uint32_t* rows,
                              uint32_t cols, const float* x, const void* act,
                              cudaStream_t stream) {
  if (nseg == 0u || nseg > static_cast<uint32_t>(kMaxSegs)) return cudaErrorInvalidValue;
  GemvSeg segs[kMaxSegs];
  for (uint32_t k = 0; k < nseg; ++k) {
    segs[k] = GemvSeg{payload[k], meta ? meta[k] : nullptr, y[k], rows[k], 0u};
  }
  GemvArgs a{};
  a.x = x;
  a.xq = static_cast<const ActChunk*>(act);
  a.cols = cols;
  switch (fmt) {
    case QG_FMT_Q4K_RAW: return launch_multi_fmt<QG_FMT_Q4K_RAW>(a, nseg, segs, stream);
    case QG_FMT_Q4K_SPLIT_PREDECODED: return launch_multi_fmt<QG_FMT_Q4K_SPLIT_PREDECODED>(a, nseg, segs, stream);
    case QG_FMT_Q4K_SPLIT_HALF: return launch_multi_fmt<QG_FMT_Q4K_SPLIT_HALF>(a, nseg, segs, stream);
    case QG_FMT_Q4K_SPLIT_COMPACT: return launch_multi_fmt<QG_FMT_Q4K_SPLIT_COMPACT>(a, nseg, segs, stream);
    case QG_FMT_Q4K_SPLIT_NATIVE: return launch_multi_fmt<QG_FMT_Q4K_SPLIT_NATIVE>(a, nseg, segs, stream);
    case QG_FMT_Q5K: return launch_multi_fmt<QG_FMT_Q5K>(a, nseg, segs, stream);
    case QG_FMT_IQ2S: return launch_multi_fmt<QG_FMT_IQ2S>(a, nseg, segs, stream);
    case QG_FMT_IQ3S: return launch_multi_fmt<QG_FMT_IQ3S>(a, nseg, segs, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qg
