// qg_aux.cu -- the small kernels around the GEMV: token argmax, the reference's
// RMSNorm/SiLU feedback kernels, bit-exact dequantization, and the layer-slice
// normalisation / gate kernels.
#include <algorithm>
#include <mutex>

#include <cooperative_groups.h>

#include "qg_formats.cuh"
#include "qg_host.h"

namespace qg {

// ---------------------------------------------------------------------------
// argmax -> token.  Lowest index wins ties; NaN never wins; the running best
// starts at -FLT_MAX with index 0, exactly like argmax_token_kernel /
// output_token_sample_kernel (decode_kernels.cu:2993-3073), so the selected index
// is the same for every input.  One CTA of 1024 threads; 16-B loads when aligned.
__device__ __forceinline__ void better(float& bv, uint32_t& bi, float v, uint32_t i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

__global__ void __launch_bounds__(1024) argmax_token_kernel(const float* __restrict__ v,
                                                            uint32_t n, uint32_t* token,
                                                            uint32_t offset, uint32_t add_token,
                                                            uint32_t modulus) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  pdl_wait();
  pdl_trigger();
  float bv = -3.4028234663852886e38f;
  uint32_t bi = 0u;
  const uint32_t tid = threadIdx.x;
  uint32_t head = 0u;
  if ((reinterpret_cast<uintptr_t>(v) & 15u) == 0u) {
    const uint32_t n4 = n >> 2;
    const float4* v4 = reinterpret_cast<const float4*>(v);
    for (uint32_t j = tid; j < n4; j += blockDim.x) {
      const float4 q = __ldg(v4 + j);
      better(bv, bi, q.x, 4u * j);
      better(bv, bi, q.y, 4u * j + 1u);
      better(bv, bi, q.z, 4u * j + 2u);
      better(bv, bi, q.w, 4u * j + 3u);
    }
    head = n4 << 2;
  }
  for (uint32_t i = head + tid; i < n; i += blockDim.x) better(bv, bi, __ldg(v + i), i);
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    better(bv, bi, ov, oi);
  }
  if ((tid & 31u) == 0u) {
    sv[tid >> 5] = bv;
    si[tid >> 5] = bi;
  }
  __syncthreads();
  if (tid < 32u) {
    const uint32_t nw = blockDim.x >> 5;
    bv = tid < nw ? sv[tid] : -3.4028234663852886e38f;
    bi = tid < nw ? si[tid] : 0u;
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
      better(bv, bi, ov, oi);
    }
    if (tid == 0u) {
      const uint32_t prev = add_token ? token[0] : 0u;
      token[0] = (bi + prev + offset) % modulus;
    }
  }
}

cudaError_t launch_argmax_token(const float* v, uint32_t n, uint32_t* token, uint32_t offset,
                                uint32_t add_token, uint32_t modulus, cudaStream_t stream) {
  return launch_k(argmax_token_kernel, 1, 1024, 0, stream, v, n, token, offset, add_token, modulus);
}

// ---------------------------------------------------------------------------
// Block-wide sum of squares of logits[0:rows] (every CTA computes it; rows is a
// stage's output length, a few thousand floats read from L2).
__device__ float block_sum_sq(const float* __restrict__ logits, uint32_t rows) {
  __shared__ float ws[32];
  float s = 0.f;
  for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) {
    const float v = __ldg(logits + r);
    s += v * v;
  }
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if ((threadIdx.x & 31u) == 0u) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32u) {
    s = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.f;
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (threadIdx.x == 0u) ws[0] = s;
  }
  __syncthreads();
  const float total = ws[0];
  __syncthreads();
  return total;
}

__device__ __forceinline__ float silu(float v) { return v * (1.0f / (1.0f + expf(-v))); }

// The reference's feedback kernels (decode_kernels.cu:122-289), one kernel with a
// mode switch; the RMS is computed once per CTA instead of once per thread.
enum FeedbackMode : uint32_t {
  kRmsnorm = 0,           // act[c] = n
  kSiluRmsnorm = 1,       // act[c] = silu(n)
  kRmsnormSiluCache = 2,  // act[c] = n, cache[c] = silu(n)
  kGatedSilu = 3,         // act[c] = cache[c % cache_cols] * n
  kCache = 4,             // cache[c] = (acc ? cache[c] : 0) + n
  kSiluCache = 5,         // cache[c] = (acc ? cache[c] : 0) + silu(n)
  kCacheGatedProduct = 6  // up[c] = (acc ? up[c] : 0) + n; act[c] = gate[c] * up[c]
};

__global__ void __launch_bounds__(256) feedback_kernel(uint32_t mode, const float* logits,
                                                       float* act, float* cache,
                                                       const float* gate, uint32_t rows,
                                                       uint32_t cols, uint32_t cache_cols,
                                                       float eps, uint32_t accumulate) {
  pdl_wait();
  pdl_trigger();
  const float sum_sq = block_sum_sq(logits, rows);
  const float inv = 1.0f / sqrtf(sum_sq / static_cast<float>(rows) + eps);
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const float n = logits[c % rows] * inv;
  switch (mode) {
    case kRmsnorm: act[c] = n; break;
    case kSiluRmsnorm: act[c] = silu(n); break;
    case kRmsnormSiluCache: act[c] = n; cache[c] = silu(n); break;
    case kGatedSilu: act[c] = cache[c % cache_cols] * n; break;
    case kCache: cache[c] = accumulate ? cache[c] + n : n; break;
    case kSiluCache: cache[c] = accumulate ? cache[c] + silu(n) : silu(n); break;
    case kCacheGatedProduct: {
      const float up = accumulate ? cache[c] + n : n;
      cache[c] = up;
      act[c] = gate[c] * up;
      break;
    }
    default: break;
  }
}

cudaError_t launch_feedback(uint32_t mode, const float* logits, float* act, float* cache,
                            const float* gate, uint32_t rows, uint32_t cols, uint32_t cache_cols,
                            float eps, uint32_t accumulate, cudaStream_t stream) {
  if (rows == 0u || cols == 0u) return cudaSuccess;  // the reference kernels return early
  const uint32_t blocks = (cols + 255u) / 256u;
  return launch_k(feedback_kernel, blocks, 256, 0, stream, mode, logits, act, cache, gate, rows, cols,
                  cache_cols, eps, accumulate);
}

// ---------------------------------------------------------------------------
// Bit-exact dequantization (one thread per value).
template <int FMT>
__global__ void dequant_kernel(const uint8_t* payload, const uint8_t* meta, uint64_t first_block,
                               uint64_t count, float* out) {
  pdl_wait();
  pdl_trigger();
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= count * 256u) return;
  out[i] = dequant_value<FMT>(payload, meta, first_block + (i >> 8), static_cast<uint32_t>(i & 255u));
}

cudaError_t launch_dequant(int fmt, const uint8_t* payload, const uint8_t* meta,
                           uint64_t first_block, uint64_t count, float* out, cudaStream_t stream) {
  const uint64_t total = count * 256u;
  const uint32_t blocks = static_cast<uint32_t>((total + 255u) / 256u);
  switch (fmt) {
#define QG_DQ(F) \
  case F: return launch_k(dequant_kernel<F>, blocks, 256, 0, stream, payload, meta, first_block, count, out);
    QG_DQ(QG_FMT_Q4K_RAW)
    QG_DQ(QG_FMT_Q4K_SPLIT_PREDECODED)
    QG_DQ(QG_FMT_Q4K_SPLIT_HALF)
    QG_DQ(QG_FMT_Q4K_SPLIT_COMPACT)
    QG_DQ(QG_FMT_Q4K_SPLIT_NATIVE)
    QG_DQ(QG_FMT_Q5K)
    QG_DQ(QG_FMT_IQ2S)
    QG_DQ(QG_FMT_IQ3S)
#undef QG_DQ
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// Layer-slice helpers (no reference counterpart): weighted RMSNorm and SiLU gate.

// y = x / sqrt(mean(x^2) + eps) * w   (one CTA; n is the hidden size)
__global__ void __launch_bounds__(1024) weighted_rmsnorm_kernel(const float* x, const float* w,
                                                                uint32_t n, float eps, float* y) {
  pdl_wait();
  pdl_trigger();
  const float sum_sq = block_sum_sq(x, n);
  const float inv = 1.0f / sqrtf(sum_sq / static_cast<float>(n) + eps);
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = x[i] * inv * w[i];
}

cudaError_t launch_weighted_rmsnorm(const float* x, const float* w, uint32_t n, float eps,
                                    float* y, cudaStream_t stream) {
  return launch_k(weighted_rmsnorm_kernel, 1, 1024, 0, stream, x, w, n, eps, y);
}

// h = silu(gate) * up
__global__ void silu_gate_kernel(const float* gate, const float* up, uint32_t n, float* h) {
  pdl_wait();
  pdl_trigger();
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) h[i] = silu(gate[i]) * up[i];
}

cudaError_t launch_silu_gate(const float* gate, const float* up, uint32_t n, float* h,
                             cudaStream_t stream) {
  return launch_k(silu_gate_kernel, (n + 255u) / 256u, 256, 0, stream, gate, up, n, h);
}

// ---------------------------------------------------------------------------
// Activation preparation: x -> one ActChunk (int8 planes + scales + sums) per 64
// columns, read by every GEMV CTA instead of re-quantizing x in each of them.  One
// warp per chunk.
__global__ void act_prepare_kernel(const float* __restrict__ x, uint32_t chunks, ActChunk* out) {
  pdl_wait();
  pdl_trigger();
  const uint32_t c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (c >= chunks) return;
  const uint32_t lane = threadIdx.x & 31u;
  const float2 v = *reinterpret_cast<const float2*>(x + 64u * c + 2u * lane);
  warp_prepare_chunk(v.x, v.y, out + c);
}

cudaError_t launch_act_prepare(const float* x, uint32_t cols, void* act, cudaStream_t stream) {
  const uint32_t chunks = cols / 64u;
  if ((reinterpret_cast<uintptr_t>(x) & 7u) != 0u) {
    // 8-B alignment is needed for the float2 loads; copy-free fallback: in-kernel path
    return cudaErrorInvalidValue;
  }
  return launch_k(act_prepare_kernel, (chunks + 3u) / 4u, 128, 0, stream, x, chunks,
                  static_cast<ActChunk*>(act));
}


// Canonical sum of squares of an RMSNorm input (every kernel that normalises a hidden
// vector uses it, so that a vector with the same bits gives the same norm whichever
// kernel -- plain or gathering -- computes it): 256 threads, thread t accumulating the
// float4 elements j = t, t + 256, ... with one fmaf per value in element order, then a
// butterfly over each warp (lane bits 16, 8, 4, 2, 1) and the eight warp sums left to
// right.  `load4(j)` returns elements 4j .. 4j + 3.
constexpr uint32_t kSumThreads = 256;

template <typename Load4>
__device__ __forceinline__ float canon_sumsq(uint32_t n4, float* ws, Load4 load4) {
  const uint32_t t = threadIdx.x;
  if (t < kSumThreads) {
    float sq = 0.f;
#pragma unroll 4
    for (uint32_t j = t; j < n4; j += kSumThreads) {
      const float4 v = load4(j);
      sq = fmaf(v.x, v.x, sq);
      sq = fmaf(v.y, v.y, sq);
      sq = fmaf(v.z, v.z, sq);
      sq = fmaf(v.w, v.w, sq);
    }
    for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    if ((t & 31u) == 0u) ws[t >> 5] = sq;
  }
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (uint32_t k = 0; k < kSumThreads / 32u; ++k) total += ws[k];
  return total;
}

// RMSNorm + int8 planes of a vector gathered from a tensor-parallel exchange, one
// thread-block cluster of up to 8 CTAs, CTA c owning elements [c n/C, (c+1) n/C).  Every
// word of every rank's slot carries the epoch it was written for: a thread issues all
// ranks' loads of an element at once and re-reads (bounded) any word that is not current
// yet.  The ranks' values are added in a pairwise tree (ranks 0+1, 2+3, ..., then the
// pairs), the same tree the row-parallel GEMV uses for the segments of a single-GPU row,
// and then added to the residual: x_out = residual + tree, the single-GPU result bit for
// bit.  A word that never becomes current makes its element NaN (and sets
// QG_ERR_WAIT_TIMEOUT), so a failed exchange cannot pass for a result.  Each CTA keeps its
// elements in shared memory; the canonical sum of squares then reads the whole vector
// from the cluster's distributed shared memory, so every CTA (and the plain
// norm_prepare_kernel on the same vector) holds the same bits.
constexpr uint32_t kMaxWordPolls = 1u << 20;  // per word, with 32 ns sleeps after the first few

__global__ void __launch_bounds__(1024) gather_norm_prepare_kernel(
    const uint64_t* buf, uint32_t* epoch, uint32_t nsrc, uint32_t stride, const float* residual,
    const float* __restrict__ w, uint32_t n, float eps, float* x_out, float* h, ActChunk* act) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) float xs[];  // this CTA's elements
  __shared__ float ws[32];
  __shared__ uint32_t gave_up;
  pdl_wait();
  pdl_trigger();
  const uint32_t cta = cluster.block_rank(), ncta = cluster.num_blocks();
  const uint32_t E = *epoch + 1u;
  const uint64_t* base = buf + (E & 1u) * static_cast<size_t>(stride);
  if (threadIdx.x == 0u) gave_up = 0u;
  cluster.sync();  // every CTA has read the epoch before it advances
  if (cta == 0u && threadIdx.x == 0u) *epoch = E;
  const uint32_t per = n / ncta, lo = cta * per;
  for (uint32_t i = lo + threadIdx.x; i < lo + per; i += blockDim.x) {
    uint64_t word[kMaxExchangeRanks];
#pragma unroll
    for (uint32_t s = 0; s < kMaxExchangeRanks; ++s) {
      if (s < nsrc) word[s] = ld_relaxed_sys_u64(base + static_cast<size_t>(s) * n + i);
    }
    float r[kMaxExchangeRanks];
#pragma unroll
    for (uint32_t s = 0; s < kMaxExchangeRanks; ++s) {
      r[s] = 0.f;
      if (s >= nsrc) continue;
      bool ok = true;
      for (uint32_t it = 0; static_cast<uint32_t>(word[s] >> 32) != E; ++it) {
        if (it == kMaxWordPolls || *reinterpret_cast<volatile uint32_t*>(&gave_up) != 0u) {
          if (atomicExch(&gave_up, 1u) == 0u) atomicOr(&g_error_word, QG_ERR_WAIT_TIMEOUT);
          ok = false;
          break;
        }
        if (it > 8u) __nanosleep(32);
        word[s] = ld_relaxed_sys_u64(base + static_cast<size_t>(s) * n + i);
      }
      r[s] = ok ? __uint_as_float(static_cast<uint32_t>(word[s])) : __uint_as_float(0x7fc00000u);
    }
#pragma unroll
    for (uint32_t step = 1; step < kMaxExchangeRanks; step <<= 1) {
#pragma unroll
      for (uint32_t s = 0; s + step < kMaxExchangeRanks; s += 2u * step) {
        if (s + step < nsrc) r[s] += r[s + step];
      }
    }
    const float v = residual != nullptr ? residual[i] + r[0] : r[0];
    x_out[i] = v;
    xs[i - lo] = v;
  }
  cluster.sync();  // every CTA's elements are in its shared memory
  const float total = canon_sumsq(n / 4u, ws, [&](uint32_t j) {
    const uint32_t owner = (4u * j) / per;
    const float* src = cluster.map_shared_rank(xs, owner);
    return *reinterpret_cast<const float4*>(src + (4u * j - owner * per));
  });
  const float inv = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
  const uint32_t lane = threadIdx.x & 31u;
  for (uint32_t c = lo / 64u + (threadIdx.x >> 5); c < (lo + per) / 64u; c += blockDim.x >> 5) {
    const uint32_t i = 64u * c + 2u * lane;
    const float v0 = xs[i - lo] * inv * w[i], v1 = xs[i + 1u - lo] * inv * w[i + 1u];
    if (h != nullptr) {
      h[i] = v0;
      h[i + 1u] = v1;
    }
    warp_prepare_chunk(v0, v1, act + c);
  }
  cluster.sync();  // no CTA leaves while another may still read its elements
}

cudaError_t launch_gather_norm_prepare(const uint64_t* buf, uint32_t* epoch, uint32_t nsrc,
                                       uint32_t stride, const float* residual, const float* w,
                                       uint32_t n, float eps, float* x_out, float* h, void* act,
                                       cudaStream_t stream) {
  if (nsrc == 0u || nsrc > kMaxExchangeRanks || buf == nullptr || epoch == nullptr ||
      x_out == nullptr || n == 0u || n % 64u != 0u) {
    return cudaErrorInvalidValue;
  }
  // CTAs: up to 8, each owning a whole number of 64-column chunks and >= 1024 elements
  uint32_t ncta = 8u;
  while (ncta > 1u && (n % (64u * ncta) != 0u || n / ncta < 1024u)) ncta >>= 1;
  const uint32_t smem = (n / ncta) * 4u;
  if (smem > 48u * 1024u) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ncta);
  cfg.blockDim = dim3(1024);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = ncta;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, gather_norm_prepare_kernel, buf, epoch, nsrc, stride, residual, w,
                            n, eps, x_out, h, static_cast<ActChunk*>(act));
}

// h = x / sqrt(mean(x^2) + eps) * w and h's int8 planes (the layer slice's and the
// decoder's RMSNorm when there is nothing to gather).  No cluster: every CTA computes the
// canonical sum of squares of the whole vector itself (it was just written, so it is read
// from L2), so all CTAs hold the same bits; then each normalises and prepares its own
// 64-column chunks, one warp per chunk.
constexpr uint32_t kNormThreads = kSumThreads;

__global__ void __launch_bounds__(kNormThreads) norm_prepare_kernel(const float* __restrict__ x,
                                                                    const float* __restrict__ w,
                                                                    uint32_t n, float eps, float* h,
                                                                    ActChunk* act) {
  __shared__ float ws[kNormThreads / 32u];
  pdl_wait();
  pdl_trigger();
  float total;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0u) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    total = canon_sumsq(n / 4u, ws, [&](uint32_t j) { return x4[j]; });
  } else {
    total = canon_sumsq(n / 4u, ws, [&](uint32_t j) {
      return make_float4(x[4u * j], x[4u * j + 1u], x[4u * j + 2u], x[4u * j + 3u]);
    });
  }
  const float inv = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t c = blockIdx.x * (kNormThreads / 32u) + warp;
  if (c < n / 64u) {
    const uint32_t i = 64u * c + 2u * lane;
    const float v0 = x[i] * inv * w[i], v1 = x[i + 1u] * inv * w[i + 1u];
    if (h != nullptr) {
      h[i] = v0;
      h[i + 1u] = v1;
    }
    warp_prepare_chunk(v0, v1, act + c);
  }
}

cudaError_t launch_norm_prepare(const float* x, const float* w, uint32_t n, float eps, float* h,
                                void* act, cudaStream_t stream) {
  if (n == 0u || n % 64u != 0u) return cudaErrorInvalidValue;
  const uint32_t chunks = n / 64u, per = kNormThreads / 32u;
  return launch_k(norm_prepare_kernel, (chunks + per - 1u) / per, kNormThreads, 0, stream, x, w, n,
                  eps, h, static_cast<ActChunk*>(act));
}

// Batched forms for the batched layer slice (row r of every [rows][n] operand).
// norm_rows_kernel: h[r] = rmsnorm(x[r]) * w with norm_prepare_kernel's sum-of-squares
// order, so each row holds the bits the single-vector kernel produces; grid (blocks, rows).
__global__ void __launch_bounds__(kNormThreads) norm_rows_kernel(const float* __restrict__ x,
                                                                 const float* __restrict__ w,
                                                                 uint32_t n, float eps, float* h) {
  __shared__ float ws[kNormThreads / 32u];
  pdl_wait();
  pdl_trigger();
  const float* xr = x + static_cast<size_t>(blockIdx.y) * n;
  float* hr = h + static_cast<size_t>(blockIdx.y) * n;
  float total;
  if ((reinterpret_cast<uintptr_t>(xr) & 15u) == 0u) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    total = canon_sumsq(n / 4u, ws, [&](uint32_t j) { return x4[j]; });
  } else {
    total = canon_sumsq(n / 4u, ws, [&](uint32_t j) {
      return make_float4(xr[4u * j], xr[4u * j + 1u], xr[4u * j + 2u], xr[4u * j + 3u]);
    });
  }
  const float inv = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    hr[i] = xr[i] * inv * w[i];
  }
}

cudaError_t launch_norm_rows(const float* x, const float* w, uint32_t n, float eps, float* h,
                             uint32_t rows, cudaStream_t stream) {
  if (n == 0u || n % 64u != 0u || rows == 0u) return cudaErrorInvalidValue;
  const uint32_t blocks = (n + kNormThreads * 4u - 1u) / (kNormThreads * 4u);
  return launch_k(norm_rows_kernel, dim3(blocks, rows), kNormThreads, 0, stream, x, w, n, eps, h);
}

// a = silu(gate) * up over `total` elements.
__global__ void silu_gate_rows_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                      size_t total, float* a) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    a[i] = silu(gate[i]) * up[i];
  }
}

cudaError_t launch_silu_gate_rows(const float* gate, const float* up, size_t total, float* a,
                                  cudaStream_t stream) {
  const uint32_t blocks = static_cast<uint32_t>(std::min<size_t>((total + 255u) / 256u, 4096u));
  return launch_k(silu_gate_rows_kernel, blocks, 256, 0, stream, gate, up, total, a);
}

// out = x + y over `total` elements (the batched slice's residual).
__global__ void add_rows_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                size_t total, float* out) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    out[i] = x[i] + y[i];
  }
}

cudaError_t launch_add_rows(const float* x, const float* y, size_t total, float* out,
                            cudaStream_t stream) {
  const uint32_t blocks = static_cast<uint32_t>(std::min<size_t>((total + 255u) / 256u, 4096u));
  return launch_k(add_rows_kernel, blocks, 256, 0, stream, x, y, total, out);
}

// a = silu(gate) * up fused with a's activation preparation (one warp per 64 columns;
// the plane scales are per 32 columns, so no cross-warp reduction is needed).
__global__ void silu_gate_prepare_kernel(const float* __restrict__ gate,
                                         const float* __restrict__ up, uint32_t n, float* a,
                                         ActChunk* act) {
  pdl_wait();
  pdl_trigger();
  const uint32_t c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (c >= n / 64u) return;
  const uint32_t i = 64u * c + 2u * (threadIdx.x & 31u);
  const float v0 = silu(gate[i]) * up[i], v1 = silu(gate[i + 1u]) * up[i + 1u];
  if (a != nullptr) {
    a[i] = v0;
    a[i + 1u] = v1;
  }
  warp_prepare_chunk(v0, v1, act + c);
}

cudaError_t launch_silu_gate_prepare(const float* gate, const float* up, uint32_t n, float* a,
                                     void* act, cudaStream_t stream) {
  const uint32_t chunks = n / 64u;
  return launch_k(silu_gate_prepare_kernel, (chunks + 3u) / 4u, 128, 0, stream, gate, up, n, a,
                  static_cast<ActChunk*>(act));
}

int device_sm_count() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace qg
