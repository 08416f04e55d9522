// qg_attn.cu -- the non-GEMV kernels of the tensor-parallel decode step (no reference
// counterpart: the reference's attention kernels are synthetic surrogates,
// runtime/kernels/decode/decode_kernels.cu:311-1136).
//
//  * Decode attention, two launches per layer: attn_split_tc_kernel (groups <= 8, tensor
//    cores) or attn_split_kernel (CUDA cores), grouped-query flash-decoding over the fp16
//    KV cache -- one CTA per (kv head, span of 64 positions) computes the span's max, sum
//    and weighted V for all q heads of the group -- then attn_combine_kernel, which merges
//    the spans of every q head in span order, normalises and writes the output and the
//    Wo GEMV's int8 planes.  The split launch also
//      - applies the rotary position embedding (adjacent pairs (2i, 2i+1), angle
//        pos * base^(-2i/head_dim)) to q as it is loaded, from a per-CTA sin/cos table
//        built while the span's loads are in flight;
//      - appends the new position: the CTA whose span holds it writes the rotated k row
//        and the v row to the cache before it reads its span.
//    (A merge inside the split launch -- the last CTA of each group of spans merging the
//    group, the last group merging the groups -- measured slower on B200 than the
//    separate combine: its chain of dependent global round trips (records, fence,
//    arrival counter, loads) left the SMs idle for 60 % of the launch.)
//  * argmax_candidate_kernel + select_token_kernel: vocab-sharded argmax (lowest index
//    wins ties).
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "qg_formats.cuh"
#include "qg_host.h"

namespace qg {

extern __device__ unsigned int g_error_word;

constexpr uint32_t kHeadDim = 128;
constexpr uint32_t kSpan = 64;       // positions per attention CTA
constexpr uint32_t kMaxGroup = 16;   // q heads per kv head

// The token position: `pos`, or *pos_dev when the step reads it from device memory
// (graphs replayed for successive tokens).
__device__ __forceinline__ uint32_t step_position(uint32_t pos, const uint32_t* pos_dev) {
  return pos_dev != nullptr ? *reinterpret_cast<const volatile uint32_t*>(pos_dev) : pos;
}

constexpr uint32_t kRec = kHeadDim + 4u;  // partial record: o[128], max, sum, 2 pad (16-B rows)

// One decode step's attention (the arguments of both split kernels).
struct AttnStep {
  const float* q;        // [n_q][128] this rank's q heads, before the rotation
  const float* k;        // [n_kv][128] the new position's k, before the rotation
  const float* v;        // [n_kv][128] the new position's v
  __half* k_cache;       // [n_kv][ctx_max][128]
  __half* v_cache;
  float* partial;        // [n_q][spans][kRec] per-span records
  const uint32_t* pos_dev;
  uint32_t G, ctx_max, pos_arg, ctx_limit, spans;
  float rope_base;
};

// Shared scratch of the prologue: the position's rotation table.
struct AttnShared {
  float cs[kHeadDim / 2u], sn[kHeadDim / 2u];
};

// The rotation table of position pos: angle i = pos * base^(-2i/head_dim).
__device__ __forceinline__ void rope_table(const AttnStep& a, uint32_t pos, AttnShared& sh) {
  const uint32_t tid = threadIdx.x;
  if (tid < kHeadDim / 2u) {
    const float inv_freq =
        powf(a.rope_base, -2.0f * static_cast<float>(tid) / static_cast<float>(kHeadDim));
    sincosf(static_cast<float>(pos) * inv_freq, &sh.sn[tid], &sh.cs[tid]);
  }
}

// Everything before the span is read: the position (or QG_ERR_POSITION) and this CTA's
// context length; in the CTA whose span holds the position, the rotation table and the
// new k (rotated) and v rows appended to the cache (`owner`).  The other CTAs build the
// table (rope_table) once their span's loads are in flight.  Returns false when the CTA
// has no positions (a span of the graph's bucket past this token's context).
__device__ __forceinline__ bool attn_prologue(const AttnStep& a, uint32_t kv, uint32_t span,
                                              AttnShared& sh, uint32_t& ctx_len, uint32_t& pos,
                                              bool& owner) {
  const uint32_t tid = threadIdx.x;
  pdl_wait();  // q, k, v come from the previous kernel
  pdl_trigger();
  pos = step_position(a.pos_arg, a.pos_dev);
  if (pos >= a.ctx_limit) {  // a position past the cache (or the graph's bucket): no work
    if (kv == 0u && span == 0u && tid == 0u) atomicOr(&g_error_word, QG_ERR_POSITION);
    return false;
  }
  ctx_len = pos + 1u;
  const uint32_t t0 = span * kSpan;
  if (t0 >= ctx_len) return false;
  owner = pos < t0 + kSpan;
  if (owner) {
    // this CTA's span holds the new position: append it before the span is read
    rope_table(a, pos, sh);
    __syncthreads();
    const size_t at = (static_cast<size_t>(kv) * a.ctx_max + pos) * kHeadDim;
    if (tid < kHeadDim / 2u) {
      const float x0 = a.k[kv * kHeadDim + 2u * tid], x1 = a.k[kv * kHeadDim + 2u * tid + 1u];
      const float cs = sh.cs[tid], sn = sh.sn[tid];
      const float r0 = x0 * cs - x1 * sn, r1 = x0 * sn + x1 * cs;
      a.k_cache[at + 2u * tid] = __float2half_rn(r0);
      a.k_cache[at + 2u * tid + 1u] = __float2half_rn(r1);
    } else if (tid < kHeadDim) {
      const uint32_t j = tid - kHeadDim / 2u;
      a.v_cache[at + 2u * j] = __float2half_rn(a.v[kv * kHeadDim + 2u * j]);
      a.v_cache[at + 2u * j + 1u] = __float2half_rn(a.v[kv * kHeadDim + 2u * j + 1u]);
    }
    __threadfence_block();
    __syncthreads();
  }
  return true;
}

// q[h][2i], q[h][2i+1] rotated by the position's angle i.
__device__ __forceinline__ float2 rope_pair(float x0, float x1, const AttnShared& sh, uint32_t i) {
  const float cs = sh.cs[i], sn = sh.sn[i];
  return make_float2(x0 * cs - x1 * sn, x0 * sn + x1 * cs);
}

// Partial attention of one kv head over positions [span*kSpan, min(+kSpan, ctx_len)),
// for its G q heads (G a compile-time group size, so every per-head loop is exact):
// the span's max score, sum of exp and exp-weighted V per head, into `partial`.
//   scores: threads (2p, 2p+1) -> position p, each over half of the head dimension with
//           its 8 K loads in flight at once, the halves combined by one shuffle;
//   values: thread d -> output dimension d, positions in blocks of 16 loads.
template <uint32_t G>
__global__ void __launch_bounds__(128) attn_split_kernel(const AttnStep a) {
  static_assert(kSpan * 2u == 128u, "two threads per position");
  __shared__ __align__(16) float qs[G][kHeadDim];
  __shared__ float p[G][kSpan];
  __shared__ float red[G][4];
  __shared__ float mx[G], sm[G];
  __shared__ __align__(16) AttnShared sh;
  const uint32_t kv = blockIdx.x, span = blockIdx.y, tid = threadIdx.x;
  const uint32_t lane = tid & 31u, warp = tid >> 5;
  const uint32_t t0 = span * kSpan;
  const float scale = rsqrtf(static_cast<float>(kHeadDim));
  const uint32_t ctx_max = a.ctx_max;
  const __half* __restrict__ k_cache = a.k_cache;
  const __half* __restrict__ v_cache = a.v_cache;
  uint32_t ctx_len = 0, step_pos = 0;
  bool owner = false;
  if (!attn_prologue(a, kv, span, sh, ctx_len, step_pos, owner)) return;
  const uint32_t n = min(kSpan, ctx_len - t0);
  if (!owner) {
    rope_table(a, step_pos, sh);
    __syncthreads();
  }
  for (uint32_t i = tid; i < G * (kHeadDim / 2u); i += blockDim.x) {  // rotated, scaled q
    const uint32_t h = i / (kHeadDim / 2u), j = i - h * (kHeadDim / 2u);
    const float* qh = a.q + (kv * G + h) * kHeadDim;
    const float2 r = rope_pair(qh[2u * j], qh[2u * j + 1u], sh, j);
    qs[h][2u * j] = r.x * scale;
    qs[h][2u * j + 1u] = r.y * scale;
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
    for (uint32_t c = 0; c < 8u; ++c) kw[c] = __ldcg(kr + c);  // L2: the new row may be this CTA's write
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
    for (uint32_t j = 0; j < 16u; ++j) vv[j] = __half2float(__ldcg(vb + static_cast<size_t>(t + j) * kHeadDim));
#pragma unroll
    for (uint32_t j = 0; j < 16u; ++j) {
#pragma unroll
      for (uint32_t h = 0; h < G; ++h) o[h] = fmaf(p[h][t + j], vv[j], o[h]);
    }
  }
  for (; t < n; ++t) {
    const float vv = __half2float(__ldcg(vb + static_cast<size_t>(t) * kHeadDim));
#pragma unroll
    for (uint32_t h = 0; h < G; ++h) o[h] = fmaf(p[h][t], vv, o[h]);
  }
  __syncthreads();
#pragma unroll
  for (uint32_t h = 0; h < G; ++h) {
    float* dst = a.partial + ((static_cast<size_t>(kv * G + h) * a.spans) + span) * kRec;
    dst[tid] = o[h];
    if (tid == 0u) {
      dst[kHeadDim] = mx[h];
      dst[kHeadDim + 1u] = sm[h];
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core split (group G <= 8 q heads per kv head), mma.sync m16n8k16 f16 -> f32.
// Four warps; warp w owns positions [16w, 16w + 16) of the span.
//  * scores S[p][h] = K[p] . q[h]: A = the warp's 16 K rows, B = the q heads (N = 8).
//    The head dimension is permuted the same way in A and B (a dot product does not
//    depend on the order of its terms): in k-step j, thread (g, t) = (lane / 4, lane % 4)
//    supplies dims 32t + 4j .. 32t + 4j + 3, so it reads 64 contiguous bytes of each of
//    its two K rows and of its q head, and no fragment needs a shuffle.  q enters as
//    q_hi + q_lo (two fp16 terms, ~2^-22 relative), so the fp16 operands add no error
//    beyond the fp16 cache.
//  * the span's per-head max and sum of exp through shared memory;
//  * weighted V: O^T[d][h] = sum_p V[p][d] P[p][h], A = V^T read with ldmatrix.trans from
//    a shared copy of the span (16-B chunk c of row p stored at chunk c ^ (p & 7), so the
//    eight rows of an 8x8 matrix fall in different banks), B = P = P_hi + P_lo.
// The four warps' O^T partials are summed in warp order into the same `partial` record
// as attn_split_kernel.

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(smem_row)));
}

__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)),
               "l"(gmem_src)
               : "memory");
}

// (hi, lo) fp16 pairs of two floats: x = hi + lo to ~2^-22 relative.
__device__ __forceinline__ void split_half2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

constexpr uint32_t kTcGroup = 8;  // q heads per kv head the tensor-core split handles (<=)

__global__ void __launch_bounds__(128) attn_split_tc_kernel(const AttnStep a) {
  static_assert(kSpan == 64u, "four warps of 16 positions");
  __shared__ __align__(128) uint8_t vs[kSpan * kHeadDim * 2u];  // the span's V, swizzled
  __shared__ float ps[4][16][9];                                 // P per warp [pos][head]
  __shared__ float ow[4][kTcGroup][kHeadDim + 4u];               // per-warp O^T [head][dim]
  __shared__ float wmax[4][kTcGroup], wsum[4][kTcGroup];
  __shared__ __align__(16) AttnShared sh;
  const uint32_t kv = blockIdx.x, span = blockIdx.y, tid = threadIdx.x;
  const uint32_t lane = tid & 31u, warp = tid >> 5, g = lane >> 2, t = lane & 3u;
  const uint32_t t0 = span * kSpan;
  const float scale = rsqrtf(static_cast<float>(kHeadDim));
  const uint32_t G = a.G, ctx_max = a.ctx_max;
  const __half* __restrict__ k_cache = a.k_cache;
  const __half* __restrict__ v_cache = a.v_cache;
  uint32_t ctx_len = 0, pos = 0;
  bool owner = false;
  if (!attn_prologue(a, kv, span, sh, ctx_len, pos, owner)) return;
  const uint32_t n = min(kSpan, ctx_len - t0);

  // V of the span -> shared memory (rows past the context are zero).
  const __half* vbase = v_cache + (static_cast<size_t>(kv) * ctx_max + t0) * kHeadDim;
  for (uint32_t i = tid; i < kSpan * 16u; i += 128u) {
    const uint32_t p = i >> 4, c = i & 15u;
    uint8_t* dst = vs + p * 256u + ((c ^ (p & 7u)) << 4);
    if (p < n) {
      cp_async_16(dst, vbase + p * kHeadDim + c * 8u);
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");

  // A fragments: K rows r0 = 16w + g and r1 = r0 + 8, dims 32t .. 32t + 31.
  const uint32_t r0 = warp * 16u + g, r1 = r0 + 8u;
  uint4 ka[4], kb[4];
  {
    const uint4* k0 = reinterpret_cast<const uint4*>(
        k_cache + (static_cast<size_t>(kv) * ctx_max + t0 + r0) * kHeadDim + 32u * t);
    const uint4* k1 = reinterpret_cast<const uint4*>(
        k_cache + (static_cast<size_t>(kv) * ctx_max + t0 + r1) * kHeadDim + 32u * t);
#pragma unroll
    for (uint32_t c = 0; c < 4u; ++c) {  // L2 loads: the new row may be this CTA's write
      ka[c] = r0 < n ? __ldcg(k0 + c) : make_uint4(0u, 0u, 0u, 0u);
      kb[c] = r1 < n ? __ldcg(k1 + c) : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  // the rotation table while the span's loads are in flight (the owner built it earlier)
  if (!owner) {
    rope_table(a, pos, sh);
    __syncthreads();
  }
  // B fragments of the scores: q head g, dims 32t .. 32t + 31 (rotated, scaled), as
  // hi + lo.
  uint32_t qh[8][2], ql[8][2];
  {
    const float4* qr = reinterpret_cast<const float4*>(
        a.q + (static_cast<size_t>(kv) * G + g) * kHeadDim + 32u * t);
#pragma unroll
    for (uint32_t j = 0; j < 8u; ++j) {
      const float4 v = g < G ? qr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      const uint32_t i0 = 16u * t + 2u * j;  // pair index of dims (32t + 4j, +1)
      const float2 r0 = rope_pair(v.x, v.y, sh, i0), r1 = rope_pair(v.z, v.w, sh, i0 + 1u);
      split_half2(r0.x * scale, r0.y * scale, qh[j][0], ql[j][0]);
      split_half2(r1.x * scale, r1.y * scale, qh[j][1], ql[j][1]);
    }
  }
  float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (uint32_t j = 0; j < 8u; ++j) {
    const uint4 x0 = ka[j >> 1], x1 = kb[j >> 1];
    const uint32_t a[4] = {(j & 1u) ? x0.z : x0.x, (j & 1u) ? x1.z : x1.x,
                           (j & 1u) ? x0.w : x0.y, (j & 1u) ? x1.w : x1.y};
    mma_f16_16816(sc, a, qh[j][0], qh[j][1]);
    mma_f16_16816(sc, a, ql[j][0], ql[j][1]);
  }
  // sc = S[r0][2t], S[r0][2t+1], S[r1][2t], S[r1][2t+1]; mask rows past the context
  if (r0 >= n) sc[0] = sc[1] = -INFINITY;
  if (r1 >= n) sc[2] = sc[3] = -INFINITY;
  float m0 = fmaxf(sc[0], sc[2]), m1 = fmaxf(sc[1], sc[3]);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
  }
  if (g == 0u) {
    wmax[warp][2u * t] = m0;
    wmax[warp][2u * t + 1u] = m1;
  }
  __syncthreads();
  const float mx0 = fmaxf(fmaxf(wmax[0][2u * t], wmax[1][2u * t]), fmaxf(wmax[2][2u * t], wmax[3][2u * t]));
  const float mx1 = fmaxf(fmaxf(wmax[0][2u * t + 1u], wmax[1][2u * t + 1u]),
                          fmaxf(wmax[2][2u * t + 1u], wmax[3][2u * t + 1u]));
  const float e0 = sc[0] == -INFINITY ? 0.f : __expf(sc[0] - mx0);
  const float e1 = sc[1] == -INFINITY ? 0.f : __expf(sc[1] - mx1);
  const float e2 = sc[2] == -INFINITY ? 0.f : __expf(sc[2] - mx0);
  const float e3 = sc[3] == -INFINITY ? 0.f : __expf(sc[3] - mx1);
  float z0 = e0 + e2, z1 = e1 + e3;
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    z0 += __shfl_xor_sync(0xffffffffu, z0, off);
    z1 += __shfl_xor_sync(0xffffffffu, z1, off);
  }
  if (g == 0u) {
    wsum[warp][2u * t] = z0;
    wsum[warp][2u * t + 1u] = z1;
  }
  ps[warp][g][2u * t] = e0;
  ps[warp][g][2u * t + 1u] = e1;
  ps[warp][g + 8u][2u * t] = e2;
  ps[warp][g + 8u][2u * t + 1u] = e3;
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();  // V in shared memory, P and the sums visible
  // B fragments of P V: P[pos 2t, 2t+1][head g] and P[pos 2t+8, 2t+9][head g].
  uint32_t ph0, pl0, ph1, pl1;
  split_half2(ps[warp][2u * t][g], ps[warp][2u * t + 1u][g], ph0, pl0);
  split_half2(ps[warp][2u * t + 8u][g], ps[warp][2u * t + 9u][g], ph1, pl1);
  const uint32_t mi = lane >> 3, rr = lane & 7u;
  const uint32_t vp = warp * 16u + rr + 8u * (mi >> 1);  // the V row this lane addresses
#pragma unroll
  for (uint32_t i = 0; i < 8u; ++i) {
    const uint32_t chunk = 2u * i + (mi & 1u);
    uint32_t a[4];
    ldmatrix_x4_trans(a, vs + vp * 256u + ((chunk ^ (vp & 7u)) << 4));
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    mma_f16_16816(o, a, ph0, ph1);
    mma_f16_16816(o, a, pl0, pl1);
    // o = O^T[16i + g][2t], [16i + g][2t+1], [16i + g + 8][2t], [16i + g + 8][2t+1]
    ow[warp][2u * t][16u * i + g] = o[0];
    ow[warp][2u * t + 1u][16u * i + g] = o[1];
    ow[warp][2u * t][16u * i + g + 8u] = o[2];
    ow[warp][2u * t + 1u][16u * i + g + 8u] = o[3];
  }
  __syncthreads();
  for (uint32_t h = 0; h < G; ++h) {
    float* dst = a.partial + ((static_cast<size_t>(kv * G + h) * a.spans) + span) * kRec;
    dst[tid] = ((ow[0][h][tid] + ow[1][h][tid]) + ow[2][h][tid]) + ow[3][h][tid];
    if (tid == 0u) {
      dst[kHeadDim] = fmaxf(fmaxf(wmax[0][h], wmax[1][h]), fmaxf(wmax[2][h], wmax[3][h]));
      dst[kHeadDim + 1u] = ((wsum[0][h] + wsum[1][h]) + wsum[2][h]) + wsum[3][h];
    }
  }
}

// Merge the spans of every q head, normalise, write attn (fp32) and its int8 planes.
// One CTA of 64 threads (two warps = the head's two 64-column chunks) per q head: the
// spans' maxima and weights are reduced in parallel, then each thread accumulates its two
// output columns over the spans with 8 loads in flight.
constexpr uint32_t kMaxSpans = 4096;

__global__ void __launch_bounds__(64) attn_combine_kernel(const float* __restrict__ partial,
                                                          uint32_t spans, uint32_t pos_arg,
                                                          const uint32_t* pos_dev, uint32_t ctx_limit,
                                                          float* out, ActChunk* act) {
  __shared__ float wgt[kMaxSpans];
  __shared__ float red[2];
  pdl_wait();
  pdl_trigger();
  const uint32_t pos = step_position(pos_arg, pos_dev);
  if (pos >= ctx_limit) return;  // the split launch recorded QG_ERR_POSITION
  const uint32_t used_spans = (pos + kSpan) / kSpan;
  const uint32_t h = blockIdx.x, tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const float* base = partial + static_cast<size_t>(h) * spans * kRec;
  float m = -INFINITY;
  for (uint32_t s = tid; s < used_spans; s += 64u) m = fmaxf(m, base[s * kRec + kHeadDim]);
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0u) red[warp] = m;
  __syncthreads();
  m = fmaxf(red[0], red[1]);
  float z = 0.f;
  for (uint32_t s = tid; s < used_spans; s += 64u) {
    const float w = __expf(base[s * kRec + kHeadDim] - m);
    wgt[s] = w;
    z = fmaf(w, base[s * kRec + kHeadDim + 1u], z);
  }
  for (int off = 16; off > 0; off >>= 1) z += __shfl_xor_sync(0xffffffffu, z, off);
  __syncthreads();  // red is reused; the weights are complete
  if (lane == 0u) red[warp] = z;
  __syncthreads();
  z = red[0] + red[1];
  float o0 = 0.f, o1 = 0.f;
  const float2* col = reinterpret_cast<const float2*>(base) + tid;  // columns 2 tid, 2 tid + 1
  constexpr uint32_t stride2 = kRec / 2u;
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
  *floats = static_cast<size_t>(n_q) * spans * kRec;
  return cudaSuccess;
}

// One layer's decode attention at the token position (`pos`, or *pos_dev with ctx_limit
// the graph's context bucket): RoPE, KV append and split in one launch, then the combine.
cudaError_t launch_attention(const float* q, const float* k, const float* v, void* k_cache,
                             void* v_cache, uint32_t n_q, uint32_t n_kv, uint32_t ctx_max,
                             uint32_t pos, const uint32_t* pos_dev, uint32_t ctx_limit,
                             float rope_base, float* partial, float* out, void* act,
                             cudaStream_t stream) {
  if (n_kv == 0u || n_q % n_kv != 0u || n_q / n_kv > kMaxGroup ||
      (ctx_max + kSpan - 1u) / kSpan > kMaxSpans || (pos_dev == nullptr && pos >= ctx_max)) {
    return cudaErrorInvalidValue;
  }
  AttnStep a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.k_cache = static_cast<__half*>(k_cache);
  a.v_cache = static_cast<__half*>(v_cache);
  a.partial = partial;
  a.pos_dev = pos_dev;
  a.G = n_q / n_kv;
  a.ctx_max = ctx_max;
  a.pos_arg = pos;
  a.ctx_limit = ctx_limit < ctx_max ? ctx_limit : ctx_max;
  a.spans = (ctx_max + kSpan - 1u) / kSpan;
  a.rope_base = rope_base;
  // the grid covers the context the launch may see: pos + 1, or the bucket
  const uint32_t reach = pos_dev != nullptr ? a.ctx_limit : pos + 1u;
  const dim3 grid(n_kv, (reach + kSpan - 1u) / kSpan);
  const bool tc = a.G <= kTcGroup && (reinterpret_cast<uintptr_t>(q) & 15u) == 0u &&
                  (reinterpret_cast<uintptr_t>(k_cache) & 15u) == 0u &&
                  (reinterpret_cast<uintptr_t>(v_cache) & 15u) == 0u;
  cudaError_t e = cudaSuccess;
  if (tc) {
    e = launch_k(attn_split_tc_kernel, grid, 128, 0, stream, a);
  } else {
    switch (a.G) {
#define QG_SPLIT(GG) \
  case GG:           \
    e = launch_k(attn_split_kernel<GG>, grid, 128, 0, stream, a); \
    break;
      QG_SPLIT(1)
      QG_SPLIT(2)
      QG_SPLIT(4)
      QG_SPLIT(8)
      QG_SPLIT(16)
#undef QG_SPLIT
      default: return cudaErrorInvalidValue;
    }
  }
  if (e != cudaSuccess) return e;
  return launch_k(attn_combine_kernel, n_q, 64, 0, stream, static_cast<const float*>(partial),
                  a.spans, pos, pos_dev, a.ctx_limit, out, static_cast<ActChunk*>(act));
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
// advance (optional): the step's position counter, incremented once the token is chosen.
__global__ void select_token_kernel(const uint32_t* cand, uint32_t ranks, uint32_t* token,
                                    uint32_t* advance) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0u || blockIdx.x != 0u) return;
  if (advance != nullptr) *advance += 1u;
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
                                uint32_t* advance, cudaStream_t stream) {
  return launch_k(select_token_kernel, 1, 32, 0, stream, cand, ranks, token, advance);
}

}  // namespace qg
