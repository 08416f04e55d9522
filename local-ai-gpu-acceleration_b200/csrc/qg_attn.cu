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
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "qg_formats.cuh"
#include "qg_host.h"

namespace qg {

constexpr uint32_t kHeadDim = 128;
constexpr uint32_t kSpan = 64;       // positions per attention CTA
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

// Partial attention of one kv head over positions [span*kSpan, min(+kSpan, ctx_len)),
// for its G q heads (G a compile-time group size, so every per-head loop is exact):
// the span's max score, sum of exp and exp-weighted V per head, into `partial`.
//   scores: threads (2p, 2p+1) -> position p, each over half of the head dimension with
//           its 8 K loads in flight at once, the halves combined by one shuffle;
//   values: thread d -> output dimension d, positions in blocks of 16 loads.
template <uint32_t G>
__global__ void __launch_bounds__(128) attn_split_kernel(const float* __restrict__ q,
                                                         const __half* __restrict__ k_cache,
                                                         const __half* __restrict__ v_cache,
                                                         uint32_t ctx_max, uint32_t ctx_len,
                                                         uint32_t spans, float* partial) {
  static_assert(kSpan * 2u == 128u, "two threads per position");
  __shared__ __align__(16) float qs[G][kHeadDim];
  __shared__ float p[G][kSpan];
  __shared__ float red[G][4];
  __shared__ float mx[G], sm[G];
  const uint32_t kv = blockIdx.x, span = blockIdx.y, tid = threadIdx.x;
  const uint32_t lane = tid & 31u, warp = tid >> 5;
  const uint32_t t0 = span * kSpan;
  const uint32_t n = ctx_len > t0 ? min(kSpan, ctx_len - t0) : 0u;
  const float scale = rsqrtf(static_cast<float>(kHeadDim));
  pdl_wait();
  pdl_trigger();
  for (uint32_t i = tid; i < G * kHeadDim; i += blockDim.x) {
    qs[i / kHeadDim][i % kHeadDim] = q[(kv * G) * kHeadDim + i] * scale;
  }
  __syncthreads();
  const uint32_t pos = tid >> 1, half = tid & 1u;
  const bool live = pos < n;
  float s[G];
#pragma unroll
  for (uint32_t h = 0; h < G; ++h) s[h] = 0.f;
  if (live) {
    const uint4* kr = reinterpret_cast<const uint4*>(
        k_cache + (static_cast<size_t>(kv) * ctx_max + t0 + pos) * kHeadDim + half * 64u);
    uint4 kw[8];
#pragma unroll
    for (uint32_t c = 0; c < 8u; ++c) kw[c] = __ldg(kr + c);
#pragma unroll
    for (uint32_t c = 0; c < 8u; ++c) {
      const __half2* hw = reinterpret_cast<const __half2*>(&kw[c]);
      float kf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(hw[e]);
        kf[2 * e] = f.x;
        kf[2 * e + 1] = f.y;
      }
#pragma unroll
      for (uint32_t h = 0; h < G; ++h) {
        const float4 qa = *reinterpret_cast<const float4*>(&qs[h][half * 64u + 8u * c]);
        const float4 qb = *reinterpret_cast<const float4*>(&qs[h][half * 64u + 8u * c + 4u]);
        s[h] = fmaf(qa.x, kf[0], s[h]);
        s[h] = fmaf(qa.y, kf[1], s[h]);
        s[h] = fmaf(qa.z, kf[2], s[h]);
        s[h] = fmaf(qa.w, kf[3], s[h]);
        s[h] = fmaf(qb.x, kf[4], s[h]);
        s[h] = fmaf(qb.y, kf[5], s[h]);
        s[h] = fmaf(qb.z, kf[6], s[h]);
        s[h] = fmaf(qb.w, kf[7], s[h]);
      }
    }
  }
#pragma unroll
  for (uint32_t h = 0; h < G; ++h) s[h] += __shfl_xor_sync(0xffffffffu, s[h], 1);  // both halves
  // per-head max and sum over the span (each position is held by two threads: the max
  // is unaffected, the sum counts the even thread only)
#pragma unroll
  for (uint32_t h = 0; h < G; ++h) {
    float m = live ? s[h] : -INFINITY;
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0u) red[h][warp] = m;
  }
  __syncthreads();
  if (tid < G) mx[tid] = fmaxf(fmaxf(red[tid][0], red[tid][1]), fmaxf(red[tid][2], red[tid][3]));
  __syncthreads();
#pragma unroll
  for (uint32_t h = 0; h < G; ++h) {
    const float e = live ? __expf(s[h] - mx[h]) : 0.f;
    if (half == 0u) p[h][pos] = e;
    float z = half == 0u ? e : 0.f;
    for (int off = 16; off > 0; off >>= 1) z += __shfl_xor_sync(0xffffffffu, z, off);
    if (lane == 0u) red[h][warp] = z;
  }
  __syncthreads();
  if (tid < G) sm[tid] = (red[tid][0] + red[tid][1]) + (red[tid][2] + red[tid][3]);
  // weighted V: thread tid -> output dimension tid; positions in blocks of 16 loads
  float o[G];
#pragma unroll
  for (uint32_t h = 0; h < G; ++h) o[h] = 0.f;
  const __half* vb = v_cache + (static_cast<size_t>(kv) * ctx_max + t0) * kHeadDim + tid;
  uint32_t t = 0;
  for (; t + 16u <= n; t += 16u) {
    float vv[16];
#pragma unroll
    for (uint32_t j = 0; j < 16u; ++j) vv[j] = __half2float(vb[static_cast<size_t>(t + j) * kHeadDim]);
#pragma unroll
    for (uint32_t j = 0; j < 16u; ++j) {
#pragma unroll
      for (uint32_t h = 0; h < G; ++h) o[h] = fmaf(p[h][t + j], vv[j], o[h]);
    }
  }
  for (; t < n; ++t) {
    const float vv = __half2float(vb[static_cast<size_t>(t) * kHeadDim]);
#pragma unroll
    for (uint32_t h = 0; h < G; ++h) o[h] = fmaf(p[h][t], vv, o[h]);
  }
  __syncthreads();
  const uint32_t stride = kHeadDim + 2u;
#pragma unroll
  for (uint32_t h = 0; h < G; ++h) {
    float* dst = partial + ((static_cast<size_t>(kv * G + h) * spans) + span) * stride;
    dst[tid] = o[h];
    if (tid == 0u) {
      dst[kHeadDim] = mx[h];
      dst[kHeadDim + 1u] = sm[h];
    }
  }
}

// Merge the spans of every q head, normalise, write attn (fp32) and its int8 planes.
// One CTA of 64 threads (two warps = the head's two 64-column chunks) per q head: the
// spans' maxima and weights are reduced in parallel, then each thread accumulates its two
// output columns over the spans with 8 loads in flight.
constexpr uint32_t kMaxSpans = 4096;

__global__ void __launch_bounds__(64) attn_combine_kernel(const float* __restrict__ partial,
                                                          uint32_t spans, uint32_t used_spans,
                                                          float* out, ActChunk* act) {
  __shared__ float wgt[kMaxSpans];
  __shared__ float red[2];
  pdl_wait();
  pdl_trigger();
  const uint32_t h = blockIdx.x, tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t stride = kHeadDim + 2u;
  const float* base = partial + static_cast<size_t>(h) * spans * stride;
  float m = -INFINITY;
  for (uint32_t s = tid; s < used_spans; s += 64u) m = fmaxf(m, base[s * stride + kHeadDim]);
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0u) red[warp] = m;
  __syncthreads();
  m = fmaxf(red[0], red[1]);
  float z = 0.f;
  for (uint32_t s = tid; s < used_spans; s += 64u) {
    const float w = __expf(base[s * stride + kHeadDim] - m);
    wgt[s] = w;
    z = fmaf(w, base[s * stride + kHeadDim + 1u], z);
  }
  for (int off = 16; off > 0; off >>= 1) z += __shfl_xor_sync(0xffffffffu, z, off);
  __syncthreads();  // red is reused; the weights are complete
  if (lane == 0u) red[warp] = z;
  __syncthreads();
  z = red[0] + red[1];
  float o0 = 0.f, o1 = 0.f;
  const float2* col = reinterpret_cast<const float2*>(base) + tid;  // columns 2 tid, 2 tid + 1
  const uint32_t stride2 = stride / 2u;
  uint32_t s = 0;
  for (; s + 8u <= used_spans; s += 8u) {
    float2 v[8];
#pragma unroll
    for (uint32_t j = 0; j < 8u; ++j) v[j] = col[static_cast<size_t>(s + j) * stride2];
#pragma unroll
    for (uint32_t j = 0; j < 8u; ++j) {
      o0 = fmaf(wgt[s + j], v[j].x, o0);
      o1 = fmaf(wgt[s + j], v[j].y, o1);
    }
  }
  for (; s < used_spans; ++s) {
    const float2 v = col[static_cast<size_t>(s) * stride2];
    o0 = fmaf(wgt[s], v.x, o0);
    o1 = fmaf(wgt[s], v.y, o1);
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
      ctx_len > ctx_max || (ctx_max + kSpan - 1u) / kSpan > kMaxSpans) {
    return cudaErrorInvalidValue;
  }
  const uint32_t spans = (ctx_max + kSpan - 1u) / kSpan;
  const uint32_t used = (ctx_len + kSpan - 1u) / kSpan;
  const uint32_t group = n_q / n_kv;
  const dim3 grid(n_kv, used);
  const __half* kc = static_cast<const __half*>(k_cache);
  const __half* vc = static_cast<const __half*>(v_cache);
  cudaError_t e;
  switch (group) {
    case 1: e = launch_k(attn_split_kernel<1>, grid, 128, 0, stream, q, kc, vc, ctx_max, ctx_len, spans, partial); break;
    case 2: e = launch_k(attn_split_kernel<2>, grid, 128, 0, stream, q, kc, vc, ctx_max, ctx_len, spans, partial); break;
    case 4: e = launch_k(attn_split_kernel<4>, grid, 128, 0, stream, q, kc, vc, ctx_max, ctx_len, spans, partial); break;
    case 8: e = launch_k(attn_split_kernel<8>, grid, 128, 0, stream, q, kc, vc, ctx_max, ctx_len, spans, partial); break;
    case 16: e = launch_k(attn_split_kernel<16>, grid, 128, 0, stream, q, kc, vc, ctx_max, ctx_len, spans, partial); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  return launch_k(attn_combine_kernel, n_q, 64, 0, stream, static_cast<const float*>(partial), spans,
                  used, out, static_cast<ActChunk*>(act));
}

// Local argmax of this rank's vocab shard -> (value bits, global index); lowest index
// wins ties.  One cluster of up to 8 CTAs, CTA c scanning [c n/C, (c+1) n/C); the CTAs'
// candidates are combined in CTA order through distributed shared memory.
__device__ __forceinline__ void better(float& bv, uint32_t& bi, float v, uint32_t i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

__global__ void __launch_bounds__(1024) argmax_candidate_kernel(const float* __restrict__ v,
                                                                uint32_t n, uint32_t offset,
                                                                uint32_t* cand) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  pdl_wait();
  pdl_trigger();
  const uint32_t c = cluster.block_rank(), nc = cluster.num_blocks();
  const uint32_t per = (n + nc - 1u) / nc, lo = c * per, hi = min(n, lo + per);
  float bv = -3.4028234663852886e38f;
  uint32_t bi = 0xffffffffu;
  for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) better(bv, bi, v[i], i);
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    better(bv, bi, ov, oi);
  }
  if ((threadIdx.x & 31u) == 0u) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0u) {
    for (uint32_t w = 1; w < (blockDim.x >> 5); ++w) better(bv, bi, sv[w], si[w]);
    sv[0] = bv;
    si[0] = bi;
  }
  cluster.sync();
  if (c == 0u && threadIdx.x == 0u) {
    float gv = -3.4028234663852886e38f;
    uint32_t gi = 0xffffffffu;
    for (uint32_t k = 0; k < nc; ++k) {
      better(gv, gi, *cluster.map_shared_rank(&sv[0], k), *cluster.map_shared_rank(&si[0], k));
    }
    if (gi == 0xffffffffu) gi = 0u;  // every value was below the initial bound (or NaN)
    cand[0] = __float_as_uint(gv);
    cand[1] = gi + offset;
  }
  cluster.sync();  // CTA 0 has read every candidate before the others leave
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
  uint32_t nc = 8u;
  while (nc > 1u && n / nc < 4096u) nc >>= 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nc);
  cfg.blockDim = dim3(1024);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = nc;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, argmax_candidate_kernel, v, n, offset, cand);
}

cudaError_t launch_select_token(const uint32_t* cand, uint32_t ranks, uint32_t* token,
                                cudaStream_t stream) {
  return launch_k(select_token_kernel, 1, 32, 0, stream, cand, ranks, token);
}

}  // namespace qg
