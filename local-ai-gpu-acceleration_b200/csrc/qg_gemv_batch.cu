// qg_gemv_batch.cu -- multi-vector quantized GEMV on the CUDA cores: the batched decode
// path below the tensor-core threshold (qg_gemm_tc.cu takes batch >= 5, the crossover
// measured on B200) and every batch of qg_gemv_batched.  No reference
// counterpart: every reference matvec kernel is batch 1
// (runtime/kernels/decode/decode_kernels.cu).
//
//   Y[b, r] = sum_c W[r, c] X[b, c]      b < NV vectors per launch (NV = 2, 4 or 8)
//
// Every weight byte is streamed from HBM once per launch and decoded once, then
// multiplied against all NV vectors, so the cost per weight is one decode plus NV
// short integer dot products instead of NV full GEMVs.
//
// Numerics.  Each launch covers one column slice of the matrix.  x is held as int16,
// one scale per (vector, slice): x~ = s * q, s = max|x over the slice| / 32767, so
// |x - x~| <= s / 2 <= 1.6e-5 ||x||_inf.  Every format's weight is a block scale times
// a small integer u (a byte), and dp2a forms two u * q products per instruction into an
// exact int32 sum per 32-column sub-block:
//   Q4_K/Q5_K  w = (d sc) u - dmin m     u = q (Q4_K high nibbles stay in place: u = 16 q,
//                                        the 1/16 goes into the scale)
//   IQ2_S      w = (d / 8) (2 s + 1) u   u = +-(2k+1), one s per 16 columns
//   IQ3_S      w = d (1 + 2 s) u         u = +-g
// (the K-quant min term uses the exact integer sum of q over the sub-block).  The
// result is sum_c w(r, c) x~(b, c) up to fp32 rounding of the per-sub-block terms, so
// |error| <= 1.6e-5 ||w_row||_1 ||x_b||_inf + fp32 accumulation -- far inside the
// 1e-3 parity bound.  Results are deterministic: fixed shuffle trees, warps summed in
// order, slices added in order.
//
// Work.  Lane l of warp w owns sub-block 32 w + l of the slice (its x values live in
// registers for the whole launch: 16 words per vector).  Persistent CTAs take units of
// q consecutive rows; warp 0 issues the first stages' copies (lane r: row r's slices,
// one 1-D bulk copy per row and array, the 16-B aligned window around the slice, L2
// evict-first) into a ring of shared-memory stages.  Per row a lane decodes its 32
// weights into eight byte words and runs 16 dp2a per vector; R = 32 / NV (at most 8)
// rows share one transposed shuffle tree; each warp posts its partial sums of a unit to a
// shared slot and arrives on that slot's mbarrier.  Unit j's epilogue -- the warps' sums
// added in warp order, scaled by the slice's x scale and written (slices after the first
// add to y: slice launches are chained on the stream), and the refill of its stage with
// unit j + S -- is done by warp j % W after its own part of unit j + 1, so no CTA-wide
// barrier stalls the warps (no producer warp either: at 8 warps a CTA keeps two per SM
// sub-partition, which leaves each thread the 255 registers the 8-vector form needs).
// Every mbarrier wait is bounded (QG_ERR_WAIT_TIMEOUT in the error word).
#include <algorithm>
#include <map>
#include <mutex>
#include <set>
#include <tuple>
#include <utility>

#include "qg_formats.cuh"
#include "qg_host.h"

namespace qg {
namespace {

constexpr uint32_t kMaxStages = 8;
constexpr uint32_t kRedSlots = 4;  // partial-sum slots in flight (units)
constexpr uint32_t kSmemLimit = 232448;  // 227 KB opt-in maximum per block

template <int NV>
__host__ __device__ constexpr uint32_t batch_max_warps() {
  return NV == 8 ? 8u : 16u;
}

struct BatchArgs {
  const uint8_t* payload;
  const uint8_t* meta;
  const float* x;         // vector v at x + v * x_stride (fp32)
  float* y;               // vector v at y + v * y_stride
  uint64_t payload_bytes; // whole arrays (a row window never reads past them)
  uint64_t meta_bytes;
  uint32_t nvec;          // live vectors (<= NV); the others are zero
  uint32_t x_stride, y_stride;
  uint32_t x_vec;         // x rows 16-B aligned: float4 loads
  uint32_t rows, kb;      // matrix rows and 256-column blocks per row
  uint32_t blk0, nblk;    // this launch's column slice: blocks [blk0, blk0 + nblk)
  uint32_t accumulate;    // 1: y += slice result (slices after the first)
  uint32_t q;             // rows per unit (= per stage)
  uint32_t units;
  uint32_t stages;
  uint32_t slot_p, slot_m;  // bytes of one row's payload / metadata slot in a stage
  uint32_t stage_bytes;
  uint32_t table_off, red_off, xs_off, stage_off;
};

// ---------------------------------------------------------------------------
// Integer dot products: a = two int16 (x), b = four bytes (weights); .lo uses bytes 0-1
// of b, .hi bytes 2-3.
__device__ __forceinline__ int dp2a_lo_u(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_u(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_lo_s(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_s(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ---------------------------------------------------------------------------
// One 32-column sub-block of one row: eight byte words (cols 4i..4i+3) and its scales.
struct SubBlock {
  uint32_t w[8];
  float mul;  // weight = mul * u (IQ2_S: times the quarter scale s0 / s1)
  float mn;   // K-quants: weight -= mn
  int s0, s1; // IQ2_S quarter scales (2 s + 1)
};

// K-quant (scale, min) of sub-block j from the 12 scale bytes (y, z, w words of the
// block header) -- get_scale_min_k4.
__device__ __forceinline__ void kq_scale_min(uint32_t y, uint32_t z, uint32_t w, uint32_t j,
                                             uint32_t& sc, uint32_t& m) {
  const uint32_t sh = 8u * (j & 3u);
  const uint32_t A = (y >> sh) & 0xffu, B = (z >> sh) & 0xffu, C = (w >> sh) & 0xffu;
  if (j < 4u) {
    sc = A & 63u;
    m = B & 63u;
  } else {
    sc = (C & 15u) | ((A >> 6) << 4);
    m = (C >> 4) | ((B >> 6) << 4);
  }
}

// Q4_K quant words of sub-block h: low nibbles of qs bytes [32 (h/2), +32) for even h,
// high nibbles (left in place, 16 q) for odd h.
__device__ __forceinline__ void q4_words(const uint8_t* qs, uint32_t h, uint32_t (&w)[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(qs);
  const uint4 b = *reinterpret_cast<const uint4*>(qs + 16);
  const uint32_t m = (h & 1u) ? 0xf0f0f0f0u : 0x0f0f0f0fu;
  w[0] = a.x & m; w[1] = a.y & m; w[2] = a.z & m; w[3] = a.w & m;
  w[4] = b.x & m; w[5] = b.y & m; w[6] = b.z & m; w[7] = b.w & m;
}

__device__ __forceinline__ void q4_header_scales(const uint4 hd, uint32_t h, SubBlock& s) {
  uint32_t sc, m;
  kq_scale_min(hd.y, hd.z, hd.w, h, sc, m);
  const float d = h2f(hd.x), dmin = h2f(hd.x >> 16);
  s.mul = d * u2f_small(sc) * ((h & 1u) ? 0.0625f : 1.0f);
  s.mn = dmin * u2f_small(m);
}

// rp / rm: this row's payload / metadata slice in shared memory; b: block in the slice;
// h: sub-block in the block.
template <int FMT>
__device__ __forceinline__ void read_sub(const uint8_t* rp, const uint8_t* rm, uint32_t b,
                                         uint32_t h, const IqTables& t, SubBlock& s);

template <>
__device__ __forceinline__ void read_sub<QG_FMT_Q4K_RAW>(const uint8_t* rp, const uint8_t*,
                                                         uint32_t b, uint32_t h, const IqTables&,
                                                         SubBlock& s) {
  const uint8_t* blk = rp + b * 144u;
  q4_words(blk + 16u + 32u * (h >> 1), h, s.w);
  q4_header_scales(*reinterpret_cast<const uint4*>(blk), h, s);
}

template <>
__device__ __forceinline__ void read_sub<QG_FMT_Q4K_SPLIT_NATIVE>(const uint8_t* rp,
                                                                  const uint8_t* rm, uint32_t b,
                                                                  uint32_t h, const IqTables&,
                                                                  SubBlock& s) {
  q4_words(rp + b * 128u + 32u * (h >> 1), h, s.w);
  q4_header_scales(*reinterpret_cast<const uint4*>(rm + b * 16u), h, s);
}

template <>
__device__ __forceinline__ void read_sub<QG_FMT_Q4K_SPLIT_PREDECODED>(const uint8_t* rp,
                                                                      const uint8_t* rm,
                                                                      uint32_t b, uint32_t h,
                                                                      const IqTables&,
                                                                      SubBlock& s) {
  q4_words(rp + b * 128u + 32u * (h >> 1), h, s.w);
  const float2 sm = *reinterpret_cast<const float2*>(rm + b * 64u + 8u * h);
  s.mul = sm.x * ((h & 1u) ? 0.0625f : 1.0f);
  s.mn = sm.y;
}

template <>
__device__ __forceinline__ void read_sub<QG_FMT_Q4K_SPLIT_HALF>(const uint8_t* rp,
                                                                const uint8_t* rm, uint32_t b,
                                                                uint32_t h, const IqTables&,
                                                                SubBlock& s) {
  q4_words(rp + b * 128u + 32u * (h >> 1), h, s.w);
  const uint32_t hm = *reinterpret_cast<const uint32_t*>(rm + b * 32u + 4u * h);
  s.mul = h2f(hm) * ((h & 1u) ? 0.0625f : 1.0f);
  s.mn = h2f(hm >> 16);
}

template <>
__device__ __forceinline__ void read_sub<QG_FMT_Q4K_SPLIT_COMPACT>(const uint8_t* rp,
                                                                   const uint8_t* rm, uint32_t b,
                                                                   uint32_t h, const IqTables&,
                                                                   SubBlock& s) {
  q4_words(rp + b * 128u + 32u * (h >> 1), h, s.w);
  const uint8_t* m = rm + b * 20u;
  const uint32_t dd = *reinterpret_cast<const uint32_t*>(m);
  s.mul = h2f(dd) * u2f_small(m[4u + h]) * ((h & 1u) ? 0.0625f : 1.0f);
  s.mn = h2f(dd >> 16) * u2f_small(m[12u + h]);
}

template <>
__device__ __forceinline__ void read_sub<QG_FMT_Q5K>(const uint8_t* rp, const uint8_t*, uint32_t b,
                                                     uint32_t h, const IqTables&, SubBlock& s) {
  const uint8_t* blk = rp + b * 176u;
  const uint4 hd = *reinterpret_cast<const uint4*>(blk);
  const uint4 h0 = *reinterpret_cast<const uint4*>(blk + 16u);
  const uint4 h1 = *reinterpret_cast<const uint4*>(blk + 32u);
  const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 48u + 32u * (h >> 1));
  const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 64u + 32u * (h >> 1));
  const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const uint32_t ns = 4u * (h & 1u);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s.w[i] = ((qw[i] >> ns) & 0x0f0f0f0fu) | (((hw[i] >> h) & 0x01010101u) << 4);
  }
  uint32_t sc, m;
  kq_scale_min(hd.y, hd.z, hd.w, h, sc, m);
  s.mul = h2f(hd.x) * u2f_small(sc);
  s.mn = h2f(hd.x >> 16) * u2f_small(m);
}

template <>
__device__ __forceinline__ void read_sub<QG_FMT_IQ2S>(const uint8_t* rp, const uint8_t*, uint32_t b,
                                                      uint32_t h, const IqTables& t, SubBlock& s) {
  const uint8_t* blk = rp + b * 82u;
  const uint32_t gl = ld_u32_a2(blk + 2u + 4u * h);
  const uint32_t sg = ld_u32_a2(blk + 34u + 4u * h);
  const uint32_t qhb = blk[66u + h], scb = blk[74u + h];
  const uint32_t h4 = spread2x4(qhb);
  uint32_t idx[4];
  idx[0] = pair_bytes<0>(gl, h4);
  idx[1] = pair_bytes<1>(gl, h4);
  idx[2] = pair_bytes<2>(gl, h4);
  idx[3] = pair_bytes<3>(gl, h4);
  const uint32_t sbs[4] = {byte_at<0>(sg), byte_at<1>(sg), byte_at<2>(sg), byte_at<3>(sg)};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint2 k2 = t.kgrid2[idx[g] * kIq2Copies];
    uint32_t m0, m1;
    sign_masks8(sbs[g], m0, m1);
    s.w[2 * g] = k2.x ^ (m0 & 0xFEFEFEFEu);
    s.w[2 * g + 1] = k2.y ^ (m1 & 0xFEFEFEFEu);
  }
  s.s0 = static_cast<int>(2u * (scb & 0x0fu) + 1u);
  s.s1 = static_cast<int>(2u * (scb >> 4) + 1u);
  s.mul = h2f(ld_u16(blk)) * 0.125f;
  s.mn = 0.f;
}

template <>
__device__ __forceinline__ void read_sub<QG_FMT_IQ3S>(const uint8_t* rp, const uint8_t*, uint32_t b,
                                                      uint32_t h, const IqTables& t, SubBlock& s) {
  const uint8_t* blk = rp + b * 110u;
  const uint32_t q0 = ld_u32_a2(blk + 2u + 8u * h), q1 = ld_u32_a2(blk + 6u + 8u * h);
  const uint32_t qhb = blk[66u + h];
  const uint32_t sg = ld_u32_a2(blk + 74u + 4u * h);
  const uint32_t nib = (blk[106u + (h >> 1)] >> (4u * (h & 1u))) & 0x0fu;
  const uint32_t hb0 = spread1x4(qhb & 0x0fu), hb1 = spread1x4(qhb >> 4);
  uint32_t idx[8];
  idx[0] = pair_bytes<0>(q0, hb0);
  idx[1] = pair_bytes<1>(q0, hb0);
  idx[2] = pair_bytes<2>(q0, hb0);
  idx[3] = pair_bytes<3>(q0, hb0);
  idx[4] = pair_bytes<0>(q1, hb1);
  idx[5] = pair_bytes<1>(q1, hb1);
  idx[6] = pair_bytes<2>(q1, hb1);
  idx[7] = pair_bytes<3>(q1, hb1);
  const uint32_t sbs[4] = {byte_at<0>(sg), byte_at<1>(sg), byte_at<2>(sg), byte_at<3>(sg)};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t m0, m1;
    sign_masks8(sbs[g], m0, m1);
    m0 &= 0xFEFEFEFEu;
    m1 &= 0xFEFEFEFEu;
    s.w[2 * g] = t.grid3[idx[2 * g] * kIq3Copies] ^ m0;
    s.w[2 * g + 1] = t.grid3[idx[2 * g + 1] * kIq3Copies] ^ m1;
  }
  s.mul = h2f(ld_u16(blk)) * u2f_small(1u + 2u * nib);
  s.mn = 0.f;
  s.s0 = s.s1 = 1;
}

template <int FMT>
struct BatchFmt {
  static constexpr uint32_t pb = FmtTraits<FMT>::payload_bytes;
  static constexpr uint32_t mb = FmtTraits<FMT>::meta_bytes;
  static constexpr bool kquant = FMT != QG_FMT_IQ2S && FMT != QG_FMT_IQ3S;
  static constexpr bool tables = !kquant;
};

// The sub-block's contribution for every vector: xw[v] its 16 x words, xs[v] the
// integer sum of its x values (K-quant min term).  The 2 NV dp2a chains advance word by
// word, so consecutive instructions are independent.
template <bool SIGNED>
__device__ __forceinline__ void dp2a_pair(uint32_t xlo, uint32_t xhi, uint32_t w, int& c0, int& c1) {
  if constexpr (SIGNED) {
    c0 = dp2a_lo_s(xlo, w, c0);
    c1 = dp2a_hi_s(xhi, w, c1);
  } else {
    c0 = dp2a_lo_u(xlo, w, c0);
    c1 = dp2a_hi_u(xhi, w, c1);
  }
}

template <int FMT, int NV>
__device__ __forceinline__ void sub_values(const SubBlock& s, const uint32_t (&xw)[NV][16],
                                           const float (&xs)[NV], float* p) {
  constexpr bool kSigned = !BatchFmt<FMT>::kquant;
  int c0[NV], c1[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) c0[v] = c1[v] = 0;
  if constexpr (FMT == QG_FMT_IQ2S) {
    int t0[NV];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int v = 0; v < NV; ++v) dp2a_pair<true>(xw[v][2 * i], xw[v][2 * i + 1], s.w[i], c0[v], c1[v]);
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      t0[v] = c0[v] + c1[v];
      c0[v] = c1[v] = 0;
    }
#pragma unroll
    for (int i = 4; i < 8; ++i) {
#pragma unroll
      for (int v = 0; v < NV; ++v) dp2a_pair<true>(xw[v][2 * i], xw[v][2 * i + 1], s.w[i], c0[v], c1[v]);
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      p[v] = s.mul * static_cast<float>(s.s0 * t0[v] + s.s1 * (c0[v] + c1[v]));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        dp2a_pair<kSigned>(xw[v][2 * i], xw[v][2 * i + 1], s.w[i], c0[v], c1[v]);
      }
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const float t = static_cast<float>(c0[v] + c1[v]);
      p[v] = BatchFmt<FMT>::kquant ? fmaf(s.mul, t, -s.mn * xs[v]) : s.mul * t;
    }
  }
}

// Sum of each of the N (<= 32) per-lane values over the warp: a transposed butterfly
// (the first log2 N exchanges, at lane offsets 16, 8, ..., trade half of the remaining
// values), then plain exchanges.  Lanes whose bits below 32 / N are zero end with the total of value
// v = sum over the transposed levels k of (bit 16 >> k of the lane) * N / 2^(k+1).
template <int N>
__device__ __forceinline__ float warp_sum_n(float (&p)[N], uint32_t lane) {
#pragma unroll
  for (int n = N, o = 16; n > 1; n >>= 1, o >>= 1) {
    const bool up = (lane & static_cast<uint32_t>(o)) != 0u;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? p[i] : p[i + n / 2];
      const float keep = up ? p[i + n / 2] : p[i];
      p[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float v = p[0];
#pragma unroll
  for (int o = 16 / N; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int N>
__device__ __forceinline__ uint32_t warp_sum_index(uint32_t lane) {
  uint32_t v = 0u;
#pragma unroll
  for (int n = N, o = 16; n > 1; n >>= 1, o >>= 1) {
    if (lane & static_cast<uint32_t>(o)) v += static_cast<uint32_t>(n / 2);
  }
  return v;
}

// Issue the copies of unit `u` (rows [u q, u q + q)) into stage `st`: per row and array
// the 16-B aligned window around the row's slice; bytes past the array's last 16-B
// boundary are copied by this thread before the arrive that publishes the stage.
__device__ __forceinline__ void window(uint64_t total, uint64_t off, uint32_t len, uint64_t& a0,
                                       uint32_t& tma_bytes) {
  a0 = off & ~15ull;
  const uint64_t end = off + len;
  const uint64_t cap = total & ~15ull;
  const uint64_t tma_end = ((end + 15ull) & ~15ull) < cap ? ((end + 15ull) & ~15ull) : cap;
  tma_bytes = tma_end > a0 ? static_cast<uint32_t>(tma_end - a0) : 0u;
}

// Issue the copies of unit `u` (rows [u q, u q + q), q <= 32) into stage `st`, lane r of
// the calling warp handling row r: per row and array the 16-B aligned window around the
// row's slice; bytes past the array's last 16-B boundary are copied by the lane itself
// before lane 0's arrive (with the stage's byte count) publishes the stage.
template <int FMT>
__device__ __forceinline__ void batch_issue(const BatchArgs& a, uint8_t* st, uint64_t* bar,
                                            uint32_t u, uint64_t policy, uint32_t lane) {
  constexpr uint32_t PB = BatchFmt<FMT>::pb, MB = BatchFmt<FMT>::mb;
  const uint32_t r0 = u * a.q;
  const uint32_t nr = min(a.q, a.rows - r0);
  uint64_t a0p = 0, a0m = 0;
  uint32_t tbp = 0, tbm = 0;
  if (lane < nr) {
    const uint64_t blk = static_cast<uint64_t>(r0 + lane) * a.kb + a.blk0;
    const uint64_t off = blk * PB, end = off + a.nblk * PB;
    window(a.payload_bytes, off, a.nblk * PB, a0p, tbp);
    uint8_t* dst = st + lane * a.slot_p;
    for (uint64_t o = a0p + tbp; o < end; ++o) dst[o - a0p] = a.payload[o];
    if (MB != 0u) {
      const uint64_t moff = blk * MB, mend = moff + a.nblk * MB;
      window(a.meta_bytes, moff, a.nblk * MB, a0m, tbm);
      uint8_t* mdst = st + a.q * a.slot_p + lane * a.slot_m;
      for (uint64_t o = a0m + tbm; o < mend; ++o) mdst[o - a0m] = a.meta[o];
    }
  }
  uint32_t total = tbp + tbm;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  __syncwarp();  // the lanes' plain copies are ordered before lane 0's (releasing) arrive
  if (lane == 0u) mbar_arrive_expect_tx(bar, total);
  __syncwarp();
  if (lane < nr) {
    if (tbp != 0u) tma_load_1d(st + lane * a.slot_p, a.payload + a0p, tbp, bar, policy);
    if (MB != 0u && tbm != 0u) {
      tma_load_1d(st + a.q * a.slot_p + lane * a.slot_m, a.meta + a0m, tbm, bar, policy);
    }
  }
}

template <int FMT, int NV>
__global__ void __launch_bounds__(32 * batch_max_warps<NV>(), 1)
    gemv_batch_kernel(const BatchArgs a) {
  constexpr uint32_t PB = BatchFmt<FMT>::pb, MB = BatchFmt<FMT>::mb;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);   // stage s filled
  uint64_t* done = full + kMaxStages;                     // partial slot k written by every warp
  uint64_t* freed = done + kRedSlots;                     // partial slot k summed (reusable)
  uint64_t* table_bar = freed + kRedSlots;
  float* red = reinterpret_cast<float*>(smem + a.red_off);
  float* xmax = reinterpret_cast<float*>(smem + a.xs_off);  // [warp][NV], then [NV] scales
  uint8_t* stages = smem + a.stage_off;

  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t nthreads = blockDim.x;
  const uint32_t W = nthreads >> 5;
  const uint32_t first = blockIdx.x, stride = gridDim.x;
  const uint32_t n_my = a.units > first ? (a.units - first + stride - 1u) / stride : 0u;
  const uint32_t S = a.stages;
  uint64_t policy = 0;

  if (tid == 0u) {
    for (uint32_t s = 0; s < S; ++s) mbar_init(&full[s], 1u);
    for (uint32_t k = 0; k < kRedSlots; ++k) {
      mbar_init(&done[k], W);
      mbar_init(&freed[k], 1u);
    }
    mbar_init(table_bar, 1u);
    fence_mbar_init();
  }
  __syncthreads();
  policy = l2_evict_first_policy();
  if (warp == 0u) {
    // Weights and tables are immutable: their copies start before the wait for the
    // previous grid.  Later stages are refilled by each unit's epilogue warp.
    if (BatchFmt<FMT>::tables && lane == 0u) {
      mbar_arrive_expect_tx(table_bar, iq_table_bytes(FMT));
      tma_load_1d(smem + a.table_off, replicated_tables<FMT>(), iq_table_bytes(FMT), table_bar);
    }
    const uint32_t pro = min(S, n_my);
    for (uint32_t i = 0; i < pro; ++i) {
      batch_issue<FMT>(a, stages + i * a.stage_bytes, &full[i], first + i * stride, policy, lane);
    }
  }

  // x of this lane's sub-block for every vector, as int16 pairs
  const uint32_t sub = 32u * warp + lane;  // sub-block of the slice
  const bool active = sub < 8u * a.nblk;
  const uint32_t b = sub >> 3, h = sub & 7u;
  const uint64_t col0 = static_cast<uint64_t>(a.blk0) * 256u + 32u * sub;
  pdl_wait();  // x (and y, when accumulating) come from earlier kernels
  pdl_trigger();

  auto load32 = [&](uint32_t v, float (&f)[32]) {
    const float* src = a.x + static_cast<uint64_t>(v) * a.x_stride + col0;
    if (a.x_vec != 0u) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 t4 = __ldg(reinterpret_cast<const float4*>(src) + i);
        f[4 * i] = t4.x; f[4 * i + 1] = t4.y; f[4 * i + 2] = t4.z; f[4 * i + 3] = t4.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) f[i] = __ldg(src + i);
    }
  };
  // slice maximum of |x| per vector
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    float m = 0.f;
    if (active && static_cast<uint32_t>(v) < a.nvec) {
      float f[32];
      load32(v, f);
#pragma unroll
      for (int i = 0; i < 32; ++i) m = fmaxf(m, fabsf(f[i]));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0u) xmax[warp * NV + v] = m;
  }
  __syncthreads();
  uint32_t xw[NV][16];
  float xs[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    float m = 0.f;
    for (uint32_t k = 0; k < W; ++k) m = fmaxf(m, xmax[k * NV + v]);
    const float inv = m > 0.f ? 32767.0f / m : 0.f;
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) xw[v][i] = 0u;
    if (active && static_cast<uint32_t>(v) < a.nvec) {
      float f[32];
      load32(v, f);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int q0 = max(-32767, min(32767, __float2int_rn(f[2 * i] * inv)));
        const int q1 = max(-32767, min(32767, __float2int_rn(f[2 * i + 1] * inv)));
        xw[v][i] = (static_cast<uint32_t>(q0) & 0xffffu) | (static_cast<uint32_t>(q1) << 16);
        sum += q0 + q1;
      }
    }
    xs[v] = static_cast<float>(sum);
  }
  if (tid < NV) {
    float m = 0.f;
    for (uint32_t k = 0; k < W; ++k) m = fmaxf(m, xmax[k * NV + tid]);
    xmax[W * NV + tid] = m > 0.f ? m / 32767.0f : 0.f;
  }
  __syncthreads();  // the slice scales, read by every epilogue warp

  const IqTables tables = iq_tables<FMT>(smem + a.table_off, lane);
  bool failed = false;
  if (BatchFmt<FMT>::tables && !mbar_wait_bounded(table_bar, 0u)) failed = true;
  // R rows share one shuffle tree of R * NV values: lane l ends with value idx (row
  // idx / NV of the group, vector idx % NV).
  constexpr int R = NV == 2 ? 8 : 4;
  constexpr int N = R * NV;
  const uint32_t idx = warp_sum_index<N>(lane);
  const uint32_t kr = idx / NV, kv = idx - kr * NV;
  const bool writer = (lane & (32u / N - 1u)) == 0u;

  // Unit j's epilogue (sum of the warps' partials in warp order, y, and the refill of
  // its stage with unit j + S) belongs to warp j % W, which does it after its own part
  // of unit j + 1: no CTA-wide barrier, warps drift apart by up to kRedSlots units.
  auto epilogue = [&](uint32_t j) -> bool {
    const uint32_t k = j % kRedSlots;
    if (!mbar_wait_bounded(&done[k], (j / kRedSlots) & 1u)) return false;
    if (j + S < n_my) {
      fence_proxy_async_smem();
      batch_issue<FMT>(a, stages + (j % S) * a.stage_bytes, &full[j % S], first + (j + S) * stride,
                       policy, lane);
    }
    const uint32_t r0 = (first + j * stride) * a.q;
    const uint32_t nr = min(a.q, a.rows - r0);
    const float* rb = red + k * (a.q * W * NV);
    for (uint32_t t = lane; t < nr * NV; t += 32u) {
      const uint32_t r = t / NV, v = t - r * NV;
      if (v >= a.nvec) continue;
      float acc = rb[(r * W) * NV + v];
      for (uint32_t w2 = 1; w2 < W; ++w2) acc += rb[(r * W + w2) * NV + v];
      acc *= xmax[W * NV + v];
      float* yp = a.y + static_cast<uint64_t>(v) * a.y_stride + r0 + r;
      *yp = a.accumulate != 0u ? *yp + acc : acc;
    }
    __syncwarp();
    if (lane == 0u) mbar_arrive(&freed[k]);
    return true;
  };

  for (uint32_t i = 0; i < n_my && !failed; ++i) {
    const uint32_t s = i % S, k = i % kRedSlots;
    const uint32_t u = first + i * stride;
    const uint32_t r0 = u * a.q;
    const uint32_t nr = min(a.q, a.rows - r0);
    if (!mbar_wait_bounded(&full[s], (i / S) & 1u)) failed = true;
    // partial slot k is free once unit i - kRedSlots has been summed
    if (!failed && i >= kRedSlots && !mbar_wait_bounded(&freed[k], (i / kRedSlots - 1u) & 1u)) {
      failed = true;
    }
    const uint8_t* st = stages + s * a.stage_bytes;
    float* rb = red + k * (a.q * W * NV);
#pragma unroll 1
    for (uint32_t g0 = 0; g0 < nr && !failed; g0 += R) {
      float p[N];
#pragma unroll
      for (int kk = 0; kk < R; ++kk) {
        const uint32_t r = g0 + kk;
        if (active && r < nr) {
          const uint64_t blk = static_cast<uint64_t>(r0 + r) * a.kb + a.blk0;
          const uint8_t* rp = st + r * a.slot_p + ((blk * PB) & 15u);
          const uint8_t* rm = st + a.q * a.slot_p + r * a.slot_m + ((blk * MB) & 15u);
          SubBlock sb;
          read_sub<FMT>(rp, rm, b, h, tables, sb);
          sub_values<FMT, NV>(sb, xw, xs, p + kk * NV);
        } else {
#pragma unroll
          for (int v = 0; v < NV; ++v) p[kk * NV + v] = 0.f;
        }
      }
      const float tot = warp_sum_n<N>(p, lane);
      if (writer && g0 + kr < nr) rb[((g0 + kr) * W + warp) * NV + kv] = tot;
    }
    __syncwarp();
    if (failed) break;
    if (lane == 0u) mbar_arrive(&done[k]);  // releases the partials and the stage reads
    if (i > 0u && (i - 1u) % W == warp && !epilogue(i - 1u)) failed = true;
  }
  if (!failed && n_my > 0u && (n_my - 1u) % W == warp && !epilogue(n_my - 1u)) failed = true;
  failed = __syncthreads_or(failed) != 0;
  if (failed && tid == 0u) {
    // Copies still in flight get a bounded chance to land before the CTA's shared memory
    // is released: the last phase issued into every stage.
    for (uint32_t s2 = 0; s2 < S && s2 < n_my; ++s2) {
      const uint32_t last = s2 + ((n_my - 1u - s2) / S) * S;
      mbar_wait_bounded(&full[s2], (last / S) & 1u);
    }
  }
}

// ---------------------------------------------------------------------------
// Host side.

struct BatchDevice {
  int sms = 0, optin = 0;
};

BatchDevice batch_device() {
  static std::mutex mu;
  static BatchDevice cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return BatchDevice{148, 227 * 1024};
  if (cache[dev].sms == 0) {
    cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  }
  return cache[dev];
}

template <typename K>
cudaError_t batch_smem_attr(K kernel, int optin) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key) == 0u) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    if (e != cudaSuccess) return e;
    done.insert(key);
  }
  return cudaSuccess;
}

template <typename K>
uint32_t batch_resident(K kernel, uint32_t threads, uint32_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, uint32_t, uint32_t, int>, uint32_t> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(reinterpret_cast<const void*>(kernel), threads, smem, dev);
  std::lock_guard<std::mutex> lock(mu);
  const auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, static_cast<int>(threads), smem) !=
          cudaSuccess || n < 1) {
    n = 1;
  }
  cache[key] = static_cast<uint32_t>(n);
  return static_cast<uint32_t>(n);
}

constexpr uint32_t round16(uint64_t v) { return static_cast<uint32_t>((v + 15u) & ~15ull); }

}  // namespace

BatchPlan plan_gemv_batch(int fmt, uint32_t nv, uint32_t rows, uint32_t cols) {
  BatchPlan p{};
  const uint32_t kb = cols / 256u;
  const uint32_t max_warps = nv > 4u ? batch_max_warps<8>() : batch_max_warps<4>();
  p.slices = (kb + 4u * max_warps - 1u) / (4u * max_warps);
  const uint32_t max_nblk = (kb + p.slices - 1u) / p.slices;
  p.warps = (max_nblk + 3u) / 4u;
  const uint32_t pb = qg_payload_bytes_per_block(fmt), mb = qg_meta_bytes_per_block(fmt);
  p.slot_p = round16(static_cast<uint64_t>(max_nblk) * pb) + 32u;
  p.slot_m = mb != 0u ? round16(static_cast<uint64_t>(max_nblk) * mb) + 32u : 0u;
  const uint32_t row_bytes = p.slot_p + p.slot_m;
  const uint32_t nvp = nv <= 2u ? 2u : nv <= 4u ? 4u : 8u;
  // units of q rows, a multiple of the R rows that share one shuffle tree, ~40 KB a stage
  const uint32_t R = nvp == 2u ? 8u : 4u;
  p.q = R * std::max(1u, std::min(16u / R, 40960u / (R * row_bytes)));
  const uint32_t table = iq_table_bytes(fmt);
  p.table_off = 256u;  // barriers first
  p.red_off = p.table_off + table;
  const uint32_t red = kRedSlots * p.q * p.warps * nvp * 4u;
  p.xs_off = p.red_off + red;
  const uint32_t xsb = (p.warps + 1u) * nvp * 4u;
  p.stage_off = (p.xs_off + xsb + 127u) & ~127u;
  p.stage_bytes = p.q * row_bytes;
  // Two CTAs per SM where the registers allow it (2..4 vectors, up to 8 warps) and three
  // stages still fit in half the shared memory; otherwise one CTA with up to 8 stages.
  const uint32_t half = kSmemLimit / 2u - 1024u;
  const bool two = nvp <= 4u && p.warps <= 8u && half > p.stage_off &&
                   (half - p.stage_off) / p.stage_bytes >= 3u;
  const uint32_t limit = two ? half : kSmemLimit;
  const uint32_t room = limit > p.stage_off ? limit - p.stage_off : 0u;
  p.stages = std::min(kMaxStages, room / p.stage_bytes);
  p.units = (rows + p.q - 1u) / p.q;
  p.smem = p.stage_off + p.stages * p.stage_bytes;
  p.ok = p.stages >= 2u ? 1u : 0u;
  return p;
}

namespace {

template <int FMT, int NV>
cudaError_t launch_batch_fmt(BatchArgs a, const BatchPlan& p, cudaStream_t stream) {
  const BatchDevice dev = batch_device();
  auto kernel = gemv_batch_kernel<FMT, NV>;
  cudaError_t e = batch_smem_attr(kernel, dev.optin);
  if (e != cudaSuccess) return e;
  const uint32_t threads = 32u * p.warps;
  const uint32_t per_sm = batch_resident(kernel, threads, p.smem);
  const uint32_t grid = std::max(1u, std::min(p.units, per_sm * static_cast<uint32_t>(dev.sms)));
  return launch_k(kernel, grid, threads, p.smem, stream, a);
}

template <int FMT>
cudaError_t launch_batch_nv(uint32_t nvp, const BatchArgs& a, const BatchPlan& p, cudaStream_t stream) {
  switch (nvp) {
    case 2: return launch_batch_fmt<FMT, 2>(a, p, stream);
    case 4: return launch_batch_fmt<FMT, 4>(a, p, stream);
    default: return launch_batch_fmt<FMT, 8>(a, p, stream);
  }
}

}  // namespace

bool gemv_batch_ok(int fmt, const uint8_t* payload, const uint8_t* meta, uint32_t rows, uint32_t cols) {
  if (fmt < 0 || fmt >= QG_FMT_COUNT || rows == 0u || cols == 0u || cols % 256u != 0u) return false;
  if ((reinterpret_cast<uintptr_t>(payload) & 15u) != 0u) return false;
  if (qg_meta_bytes_per_block(fmt) != 0u && (reinterpret_cast<uintptr_t>(meta) & 15u) != 0u) return false;
  return plan_gemv_batch(fmt, 8u, rows, cols).ok != 0u && plan_gemv_batch(fmt, 4u, rows, cols).ok != 0u;
}

cudaError_t launch_gemv_batch(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                              float* y, uint32_t nvec, uint32_t x_stride, uint32_t y_stride,
                              uint32_t rows, uint32_t cols, cudaStream_t stream) {
  if (nvec == 0u || nvec > 8u) return cudaErrorInvalidValue;
  const BatchPlan p = plan_gemv_batch(fmt, nvec, rows, cols);
  if (!p.ok) return cudaErrorInvalidValue;
  const uint32_t kb = cols / 256u;
  const uint32_t nvp = nvec <= 2u ? 2u : nvec <= 4u ? 4u : 8u;
  BatchArgs a{};
  a.payload = payload;
  a.meta = meta;
  a.x = x;
  a.y = y;
  a.payload_bytes = static_cast<uint64_t>(rows) * kb * qg_payload_bytes_per_block(fmt);
  a.meta_bytes = static_cast<uint64_t>(rows) * kb * qg_meta_bytes_per_block(fmt);
  a.nvec = nvec;
  a.x_stride = x_stride;
  a.y_stride = y_stride;
  a.x_vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0u && x_stride % 4u == 0u) ? 1u : 0u;
  a.rows = rows;
  a.kb = kb;
  a.q = p.q;
  a.units = p.units;
  a.stages = p.stages;
  a.slot_p = p.slot_p;
  a.slot_m = p.slot_m;
  a.stage_bytes = p.stage_bytes;
  a.table_off = p.table_off;
  a.red_off = p.red_off;
  a.xs_off = p.xs_off;
  a.stage_off = p.stage_off;
  // Column slices, one launch each, chained on the stream (y = slice 0, then y += ...).
  const uint32_t base = kb / p.slices, extra = kb % p.slices;
  uint32_t blk0 = 0;
  for (uint32_t k = 0; k < p.slices; ++k) {
    a.blk0 = blk0;
    a.nblk = base + (k < extra ? 1u : 0u);
    a.accumulate = k > 0u ? 1u : 0u;
    blk0 += a.nblk;
    cudaError_t e = cudaSuccess;
    switch (fmt) {
      case QG_FMT_Q4K_RAW: e = launch_batch_nv<QG_FMT_Q4K_RAW>(nvp, a, p, stream); break;
      case QG_FMT_Q4K_SPLIT_PREDECODED: e = launch_batch_nv<QG_FMT_Q4K_SPLIT_PREDECODED>(nvp, a, p, stream); break;
      case QG_FMT_Q4K_SPLIT_HALF: e = launch_batch_nv<QG_FMT_Q4K_SPLIT_HALF>(nvp, a, p, stream); break;
      case QG_FMT_Q4K_SPLIT_COMPACT: e = launch_batch_nv<QG_FMT_Q4K_SPLIT_COMPACT>(nvp, a, p, stream); break;
      case QG_FMT_Q4K_SPLIT_NATIVE: e = launch_batch_nv<QG_FMT_Q4K_SPLIT_NATIVE>(nvp, a, p, stream); break;
      case QG_FMT_Q5K: e = launch_batch_nv<QG_FMT_Q5K>(nvp, a, p, stream); break;
      case QG_FMT_IQ2S: e = launch_batch_nv<QG_FMT_IQ2S>(nvp, a, p, stream); break;
      case QG_FMT_IQ3S: e = launch_batch_nv<QG_FMT_IQ3S>(nvp, a, p, stream); break;
      default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Y = W X for `batch` vectors (X [batch][cols], Y [batch][rows]): groups of up to 8
// vectors, each group one pass over the weights (a single vector takes the batch-1
// GEMV); packs the multi-vector kernel cannot stage go vector by vector.
cudaError_t launch_gemv_vectors(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                                float* y, uint32_t batch, uint32_t rows, uint32_t cols,
                                cudaStream_t stream) {
  const bool multi = gemv_batch_ok(fmt, payload, meta, rows, cols);
  for (uint32_t v0 = 0; v0 < batch;) {
    const uint32_t nv = multi ? std::min(8u, batch - v0) : 1u;
    const float* xv = x + static_cast<uint64_t>(v0) * cols;
    float* yv = y + static_cast<uint64_t>(v0) * rows;
    const cudaError_t e =
        nv == 1u ? launch_gemv(fmt, payload, meta, xv, nullptr, yv, nullptr, nullptr, nullptr, 0u, 0u,
                               0u, rows, cols, stream)
                 : launch_gemv_batch(fmt, payload, meta, xv, yv, nv, cols, rows, rows, cols, stream);
    if (e != cudaSuccess) return e;
    v0 += nv;
  }
  return cudaSuccess;
}

}  // namespace qg
