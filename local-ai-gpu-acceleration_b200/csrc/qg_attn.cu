// qg_attn.cu -- the non-GEMV kernels of the tensor-parallel decode step (no reference
// counterpart: the reference's attention kernels are synthetic surrogates,
// runtime/kernels/decode/decode_kernels.cu:311-1136).
//
//  * rope_append_kernel: rotary position embedding of this rank's q and k heads
//    (adjacent pairs (2i, 2i+1), angle pos * base^(-2i/head_dim)), then k and v of the
//    new position written to the fp16 KV cache.
//  * attn_split_kernel + attn_combine_kernel: grouped-query decode attention over the
//    fp16 cache (flash-decoding: one CTA per (kv head, span of positions) computes the
//    span's max, sum and weighted V for all q heads of the group; the combine merges
//    the spans, normalises and emits the Wo GEMV's int8 planes).
//  * argmax_candidate_kernel + select_token_kernel: vocab-sharded argmax (lowest index
//    wins ties).
#include <cuda_fp16.h>

#include "qg_formats.cuh"
#include "qg_host.h"

namespace qg {

constexpr uint32_t kHeadDim = 128;
constexpr uint32_t kSpan = 128;      // positions per attention CTA
constexpr uint32_t kMaxGroup = 16;   // q heads per kv head

__global__ void rope_append_kernel(float* q, float* k, const float* v, __half* k_cache,
                                   __half* v_cache, uint32_t n_q, uint32_t n_kv, uint32_t ctx_max,
                                   uint32_t pos, float rope_base) {
  pdl_wait();
  pdl_trigger();
  // one thread per rotation pair of one head (q heads first, then k heads), plus the
  // v copy done by the k-head threads
  const uint32_t pairs = kHeadDim / 2u;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t head = i / pairs, j = i - head * pairs;
  if (head >= n_q + n_kv) return;
  const float inv_freq = powf(rope_base, -2.0f * static_cast<float>(j) / static_cast<float>(kHeadDim));
  float sn, cs;
  sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
  float* base = head < n_q ? q + head * kHeadDim : k + (head - n_q) * kHeadDim;
  const float a = base[2u * j], b = base[2u * j + 1u];
  const float ra = a * cs - b * sn, rb = a * sn + b * cs;
  base[2u * j] = ra;
  base[2u * j + 1u] = rb;
  if (head >= n_q) {
    const uint32_t kv = head - n_q;
    const size_t at = (static_cast<size_t>(kv) * ctx_max + pos) * kHeadDim + 2u * j;
    k_cache[at] = __float2half_rn(ra);
    k_cache[at + 1u] = __float2half_rn(rb);
    v_cache[at] = __float2half_rn(v[kv * kHeadDim + 2u * j]);
    v_cache[at + 1u] = __float2half_rn(v[kv * kHeadDim + 2u * j + 1u]);
  }
}

cudaError_t launch_rope_append(float* q, float* k, const float* v, void* k_cache, void* v_cache,
                               uint32_t n_q, uint32_t n_kv, uint32_t ctx_max, uint32_t pos,
                               float rope_base, cudaStream_t stream) {
  const uint32_t threads = (n_q + n_kv) * (kHeadDim / 2u);
  return launch_k(rope_append_kernel, (threads + 127u) / 128u, 128, 0, stream, q, k, v,
                  static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), n_q, n_kv, ctx_max,
                  pos, rope_base);
}

// Partial attention of one kv head over positions [span*kSpan, min(+kSpan, ctx_len)).
// Thread t scores position t for every q head of the group; thread d then accumulates
// output dimension d.  Writes, per (q head, span): kHeadDim weighted-V sums, the max
// score and the sum of exp(score - max).
__global__ void __launch_bounds__(128) attn_split_kernel(const float* __restrict__ q,
                                                         const __half* __restrict__ k_cache,
                                                         const __half* __restrict__ v_cache,
                                                         uint32_t group, uint32_t ctx_max,
                                                         uint32_t ctx_len, uint32_t spans,
                                                         float* partial) {
  __shared__ float qs[kMaxGroup][kHeadDim];
  __shared__ float p[kMaxGroup][kSpan];
  __shared__ float red[kMaxGroup][4];
  __shared__ float mx[kMaxGroup], sm[kMaxGroup];
  const uint32_t kv = blockIdx.x, span = blockIdx.y, tid = threadIdx.x;
  const uint32_t t0 = span * kSpan;
  const uint32_t n = ctx_len > t0 ? min(kSpan, ctx_len - t0) : 0u;
  const float scale = rsqrtf(static_cast<float>(kHeadDim));
  pdl_wait();
  pdl_trigger();
  for (uint32_t i = tid; i < group * kHeadDim; i += blockDim.x) {
    qs[i / kHeadDim][i % kHeadDim] = q[(kv * group) * kHeadDim + i] * scale;
  }
  __syncthreads();
  // scores: thread tid -> position t0 + tid
  float s[kMaxGroup];
#pragma unroll
  for (uint32_t h = 0; h < kMaxGroup; ++h) s[h] = 0.f;
  if (tid < n) {
    const uint4* kr = reinterpret_cast<const uint4*>(k_cache + (static_cast<size_t>(kv) * ctx_max + t0 + tid) * kHeadDim);
#pragma unroll 4
    for (uint32_t c = 0; c < kHeadDim / 8u; ++c) {
      const uint4 w = __ldg(kr + c);
      const __half2* hw = reinterpret_cast<const __half2*>(&w);
      float kvv[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(hw[e]);
        kvv[2 * e] = f.x;
        kvv[2 * e + 1] = f.y;
      }
#pragma unroll
      for (uint32_t h = 0; h < kMaxGroup; ++h) {
        if (h < group) {
#pragma unroll
          for (int e = 0; e < 8; ++e) s[h] = fmaf(qs[h][8u * c + e], kvv[e], s[h]);
        }
      }
    }
  }
  // per-head max and sum over the span
  const uint32_t lane = tid & 31u, warp = tid >> 5;
#pragma unroll
  for (uint32_t h = 0; h < kMaxGroup; ++h) {
    if (h >= group) break;
    float m = tid < n ? s[h] : -INFINITY;
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0u) red[h][warp] = m;
  }
  __syncthreads();
  if (tid < group) mx[tid] = fmaxf(fmaxf(red[tid][0], red[tid][1]), fmaxf(red[tid][2], red[tid][3]));
  __syncthreads();
#pragma unroll
  for (uint32_t h = 0; h < kMaxGroup; ++h) {
    if (h >= group) break;
    const float e = tid < n ? __expf(s[h] - mx[h]) : 0.f;
    p[h][tid] = e;
    float z = e;
    for (int off = 16; off > 0; off >>= 1) z += __shfl_xor_sync(0xffffffffu, z, off);
    if (lane == 0u) red[h][warp] = z;
  }
  __syncthreads();
  if (tid < group) sm[tid] = (red[tid][0] + red[tid][1]) + (red[tid][2] + red[tid][3]);
  // weighted V: thread tid -> output dimension tid
  float o[kMaxGroup];
#pragma unroll
  for (uint32_t h = 0; h < kMaxGroup; ++h) o[h] = 0.f;
  const __half* vb = v_cache + (static_cast<size_t>(kv) * ctx_max + t0) * kHeadDim + tid;
  for (uint32_t t = 0; t < n; ++t) {
    const float vv = __half2float(vb[static_cast<size_t>(t) * kHeadDim]);
#pragma unroll
    for (uint32_t h = 0; h < kMaxGroup; ++h) {
      if (h < group) o[h] = fmaf(p[h][t], vv, o[h]);
    }
  }
  __syncthreads();
  const uint32_t stride = kHeadDim + 2u;
  for (uint32_t h = 0; h < group; ++h) {
    float* dst = partial + ((static_cast<size_t>(kv * group + h) * spans) + span) * stride;
    dst[tid] = o[h];
    if (tid == 0u) {
      dst[kHeadDim] = mx[h];
      dst[kHeadDim + 1u] = sm[h];
    }
  }
}

// Merge the spans of every q head, normalise, write attn (fp32) and its int8 planes.
// One CTA of 64 threads (two warps = the head's two 64-column chunks) per q head.
__global__ void __launch_bounds__(64) attn_combine_kernel(const float* __restrict__ partial,
                                                          uint32_t spans, uint32_t used_spans,
                                                          float* out, ActChunk* act) {
  pdl_wait();
  pdl_trigger();
  const uint32_t h = blockIdx.x, tid = threadIdx.x;
  const uint32_t stride = kHeadDim + 2u;
  const float* base = partial + static_cast<size_t>(h) * spans * stride;
  float m = -INFINITY;
  for (uint32_t s = 0; s < used_spans; ++s) m = fmaxf(m, base[s * stride + kHeadDim]);
  float z = 0.f, o0 = 0.f, o1 = 0.f;
  for (uint32_t s = 0; s < used_spans; ++s) {
    const float* ps = base + s * stride;
    const float w = __expf(ps[kHeadDim] - m);
    z = fmaf(w, ps[kHeadDim + 1u], z);
    o0 = fmaf(w, ps[2u * tid], o0);
    o1 = fmaf(w, ps[2u * tid + 1u], o1);
  }
  const float inv = 1.0f / z;
  o0 *= inv;
  o1 *= inv;
  out[h * kHeadDim + 2u * tid] = o0;
  out[h * kHeadDim + 2u * tid + 1u] = o1;
  warp_prepare_chunk(o0, o1, act + h * 2u + (tid >> 5));
}

cudaError_t attn_partial_floats(uint32_t n_q, uint32_t ctx_max, size_t* floats) {
  const uint32_t spans = (ctx_max + kSpan - 1u) / kSpan;
  *floats = static_cast<size_t>(n_q) * spans * (kHeadDim + 2u);
  return cudaSuccess;
}

cudaError_t launch_attention(const float* q, const void* k_cache, const void* v_cache,
                             uint32_t n_q, uint32_t n_kv, uint32_t ctx_max, uint32_t ctx_len,
                             float* partial, float* out, void* act, cudaStream_t stream) {
  if (n_kv == 0u || n_q % n_kv != 0u || n_q / n_kv > kMaxGroup || ctx_len == 0u ||
      ctx_len > ctx_max) {
    return cudaErrorInvalidValue;
  }
  const uint32_t spans = (ctx_max + kSpan - 1u) / kSpan;
  const uint32_t used = (ctx_len + kSpan - 1u) / kSpan;
  cudaError_t e = launch_k(attn_split_kernel, dim3(n_kv, used), 128, 0, stream, q,
                           static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache),
                           n_q / n_kv, ctx_max, ctx_len, spans, partial);
  if (e != cudaSuccess) return e;
  return launch_k(attn_combine_kernel, n_q, 64, 0, stream, static_cast<const float*>(partial), spans,
                  used, out, static_cast<ActChunk*>(act));
}

// Local argmax of this rank's vocab shard -> (value bits, global index).
__global__ void __launch_bounds__(1024) argmax_candidate_kernel(const float* __restrict__ v,
                                                                uint32_t n, uint32_t offset,
                                                                uint32_t* cand) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  pdl_wait();
  pdl_trigger();
  float bv = -3.4028234663852886e38f;
  uint32_t bi = 0u;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float x = v[i];
    if (x > bv || (x == bv && i < bi)) {
      bv = x;
      bi = i;
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31u) == 0u) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0u) {
    for (uint32_t w = 1; w < (blockDim.x >> 5); ++w) {
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
        bv = sv[w];
        bi = si[w];
      }
    }
    cand[0] = __float_as_uint(bv);
    cand[1] = bi + offset;
  }
}

// token = global argmax over the gathered (value, index) candidates of all ranks.
__global__ void select_token_kernel(const uint32_t* cand, uint32_t ranks, uint32_t* token) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0u || blockIdx.x != 0u) return;
  float bv = __uint_as_float(cand[0]);
  uint32_t bi = cand[1];
  for (uint32_t r = 1; r < ranks; ++r) {
    const float v = __uint_as_float(cand[2u * r]);
    const uint32_t i = cand[2u * r + 1u];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
  token[0] = bi;
}

cudaError_t launch_argmax_candidate(const float* v, uint32_t n, uint32_t offset, uint32_t* cand,
                                    cudaStream_t stream) {
  return launch_k(argmax_candidate_kernel, 1, 1024, 0, stream, v, n, offset, cand);
}

cudaError_t launch_select_token(const uint32_t* cand, uint32_t ranks, uint32_t* token,
                                cudaStream_t stream) {
  return launch_k(select_token_kernel, 1, 32, 0, stream, cand, ranks, token);
}

}  // namespace qg
