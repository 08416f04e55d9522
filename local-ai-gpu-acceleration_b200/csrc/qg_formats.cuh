// qg_formats.cuh -- per-format quant readers for the sm_100a decode kernels.
//
// Two readers per format:
//  * dequant_value<FMT>: one value, same arithmetic and order as the reference's
//    CPU decode (runtime/apps/mixed_sequence_benchmark_runner/main.cpp:1086-1259,
//    device twins decode_kernels.cu:1504-1728) with explicit _rn operations so
//    nvcc cannot contract them -- bit-identical fp32 output.
//  * chunk_dot<FMT>: the GEMV inner product of one 64-column chunk of one row,
//    reading the row's bytes from shared memory.  It uses the factorised form
//    sum_sub (d*scale) * sum(q*x) - (dmin*min) * sum(x) with packed f32x2 FMAs, so
//    it agrees with the reference within fp32 reassociation error.
//
// A 64-column chunk c of a row covers columns [64c, 64c+64): for the K-quants the
// low/high nibbles of qs[32*(c%4) .. +32) of block c/4, for the IQ formats the two
// 32-value sub-blocks 2*(c%4), 2*(c%4)+1 of block c/4.  The thread that owns chunk c
// keeps x[64c .. 64c+64) in registers as xa (first 32) and xb (last 32).
#pragma once

#include "qg_common.cuh"

namespace qg {

// ---------------------------------------------------------------------------
// Codebooks.  Copied from global memory into each CTA's shared memory by the
// IQ kernels; the dequant kernel reads them from global memory directly.
extern __device__ uint16_t g_iq2s_kgrid[1024];
extern __device__ uint32_t g_iq3s_grid[512];

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
  return static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(p));
}
// Four bytes from a 2-byte aligned address.
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t* p) {
  return ld_u16(p) | (ld_u16(p + 2) << 16u);
}
__device__ __forceinline__ uint32_t ld_bytes_u16(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8u);
}

// ---------------------------------------------------------------------------
// Bit-exact single-value readers (global memory, byte loads).

template <int FMT>
__device__ __forceinline__ float dequant_value(const uint8_t* payload, const uint8_t* meta,
                                               uint64_t bi, uint32_t v);

// Q4_K (raw and split packs): main.cpp:1133-1171; raw 144-B block = split-native
// with meta = block[0:16], payload = block[16:144].
__device__ __forceinline__ float q4k_value(int fmt, const uint8_t* pb, const uint8_t* mb,
                                           uint32_t v) {
  const uint32_t g64 = v >> 6u, w64 = v & 63u, lane = w64 & 31u;
  const bool hi = w64 >= 32u;
  const uint32_t pair = g64 * 2u + (hi ? 1u : 0u);
  const uint32_t packed = pb[g64 * 32u + lane];
  const float quant = static_cast<float>(hi ? (packed >> 4u) : (packed & 0x0fu));
  if (fmt == QG_FMT_Q4K_SPLIT_PREDECODED) {
    const float s = __uint_as_float(ld_bytes_u16(mb + pair * 8u) |
                                    (ld_bytes_u16(mb + pair * 8u + 2u) << 16u));
    const float m = __uint_as_float(ld_bytes_u16(mb + pair * 8u + 4u) |
                                    (ld_bytes_u16(mb + pair * 8u + 6u) << 16u));
    return __fsub_rn(__fmul_rn(s, quant), m);
  }
  if (fmt == QG_FMT_Q4K_SPLIT_HALF) {
    const float s = h2f(ld_bytes_u16(mb + pair * 4u));
    const float m = h2f(ld_bytes_u16(mb + pair * 4u + 2u));
    return __fsub_rn(__fmul_rn(s, quant), m);
  }
  const float d = h2f(ld_bytes_u16(mb));
  const float dmin = h2f(ld_bytes_u16(mb + 2u));
  uint32_t sc, mn;
  if (fmt == QG_FMT_Q4K_SPLIT_COMPACT) {
    sc = mb[4u + pair];
    mn = mb[12u + pair];
  } else {
    const uint8_t* s = mb + 4u;
    const uint32_t s0 = s[0] | (s[1] << 8) | (s[2] << 16) | (static_cast<uint32_t>(s[3]) << 24);
    const uint32_t s1 = s[4] | (s[5] << 8) | (s[6] << 16) | (static_cast<uint32_t>(s[7]) << 24);
    const uint32_t s2 = s[8] | (s[9] << 8) | (s[10] << 16) | (static_cast<uint32_t>(s[11]) << 24);
    scale_min_k4(pair, s0, s1, s2, sc, mn);
  }
  return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), quant),
                   __fmul_rn(dmin, static_cast<float>(mn)));
}

template <>
__device__ __forceinline__ float dequant_value<QG_FMT_Q4K_RAW>(const uint8_t* payload,
                                                               const uint8_t*, uint64_t bi,
                                                               uint32_t v) {
  const uint8_t* blk = payload + bi * 144u;
  return q4k_value(QG_FMT_Q4K_SPLIT_NATIVE, blk + 16, blk, v);
}
#define QG_SPLIT_DEQUANT(F)                                                            \
  template <>                                                                          \
  __device__ __forceinline__ float dequant_value<F>(const uint8_t* payload,            \
                                                    const uint8_t* meta, uint64_t bi,  \
                                                    uint32_t v) {                      \
    return q4k_value(F, payload + bi * 128u, meta + bi * FmtTraits<F>::meta_bytes, v);   \
  }
QG_SPLIT_DEQUANT(QG_FMT_Q4K_SPLIT_PREDECODED)
QG_SPLIT_DEQUANT(QG_FMT_Q4K_SPLIT_HALF)
QG_SPLIT_DEQUANT(QG_FMT_Q4K_SPLIT_COMPACT)
QG_SPLIT_DEQUANT(QG_FMT_Q4K_SPLIT_NATIVE)
#undef QG_SPLIT_DEQUANT

// Q5_K: main.cpp:1231-1259.
template <>
__device__ __forceinline__ float dequant_value<QG_FMT_Q5K>(const uint8_t* payload, const uint8_t*,
                                                           uint64_t bi, uint32_t v) {
  const uint8_t* blk = payload + bi * 176u;
  const float d = h2f(ld_bytes_u16(blk));
  const float dmin = h2f(ld_bytes_u16(blk + 2));
  const uint8_t* s = blk + 4;
  const uint32_t s0 = s[0] | (s[1] << 8) | (s[2] << 16) | (static_cast<uint32_t>(s[3]) << 24);
  const uint32_t s1 = s[4] | (s[5] << 8) | (s[6] << 16) | (static_cast<uint32_t>(s[7]) << 24);
  const uint32_t s2 = s[8] | (s[9] << 8) | (s[10] << 16) | (static_cast<uint32_t>(s[11]) << 24);
  const uint32_t g64 = v >> 6u, w64 = v & 63u, lane = w64 & 31u;
  const bool hi = w64 >= 32u;
  uint32_t sc, mn;
  scale_min_k4(g64 * 2u + (hi ? 1u : 0u), s0, s1, s2, sc, mn);
  const uint32_t packed = blk[48u + g64 * 32u + lane];
  const uint32_t low = hi ? (packed >> 4u) : (packed & 0x0fu);
  const uint32_t mask = (hi ? 2u : 1u) << (g64 * 2u);
  const uint32_t quant = low + ((blk[16u + lane] & mask) ? 16u : 0u);
  return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(quant)),
                   __fmul_rn(dmin, static_cast<float>(mn)));
}

// IQ2_S: main.cpp:1173-1194.
template <>
__device__ __forceinline__ float dequant_value<QG_FMT_IQ2S>(const uint8_t* payload,
                                                            const uint8_t*, uint64_t bi,
                                                            uint32_t v) {
  const uint8_t* blk = payload + bi * 82u;
  const uint32_t ib32 = v >> 5u, w32 = v & 31u, group = w32 >> 3u, lane = w32 & 7u;
  const float d = h2f(ld_bytes_u16(blk));
  const uint8_t* qs = blk + 2;
  const uint32_t go = ib32 * 4u + group;
  const uint32_t idx = qs[go] | ((static_cast<uint32_t>(blk[66u + ib32]) << (8u - 2u * group)) & 0x300u);
  const uint32_t grid = 2u * ((static_cast<uint32_t>(g_iq2s_kgrid[idx]) >> (2u * lane)) & 3u) + 1u;
  const uint32_t sb = blk[74u + ib32];
  const uint32_t nib = group < 2u ? (sb & 0x0fu) : (sb >> 4u);
  const float scale = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, static_cast<float>(nib))), 0.25f);
  const bool neg = (qs[32u + go] & (1u << lane)) != 0u;
  return __fmul_rn(__fmul_rn(scale, static_cast<float>(grid)), neg ? -1.0f : 1.0f);
}

// IQ3_S: main.cpp:1196-1221.
template <>
__device__ __forceinline__ float dequant_value<QG_FMT_IQ3S>(const uint8_t* payload,
                                                            const uint8_t*, uint64_t bi,
                                                            uint32_t v) {
  const uint8_t* blk = payload + bi * 110u;
  const uint32_t ib32 = v >> 5u, w32 = v & 31u, group = w32 >> 3u, lane = w32 & 7u;
  const uint32_t pair = lane >> 2u, glane = lane & 3u;
  const float d = h2f(ld_bytes_u16(blk));
  const uint32_t sel = ib32 * 8u + group * 2u + pair;
  const uint32_t hb = (static_cast<uint32_t>(blk[66u + ib32]) >> (2u * group + pair)) & 1u;
  const uint32_t idx = blk[2u + sel] | (hb << 8u);
  const uint32_t grid = (g_iq3s_grid[idx] >> (8u * glane)) & 0xffu;
  const uint32_t sb = blk[106u + (ib32 >> 1u)];
  const uint32_t nib = (ib32 & 1u) == 0u ? (sb & 0x0fu) : (sb >> 4u);
  const float scale = __fmul_rn(d, static_cast<float>(1u + 2u * nib));
  const bool neg = (blk[74u + ib32 * 4u + group] & (1u << lane)) != 0u;
  return __fmul_rn(__fmul_rn(scale, static_cast<float>(grid)), neg ? -1.0f : 1.0f);
}

// ---------------------------------------------------------------------------
// GEMV chunk readers (shared memory).

struct ChunkX {
  float2 a[16];  // x[64c + 0 .. 31]
  float2 b[16];  // x[64c + 32 .. 63]
  float sa, sb;  // sum of a, sum of b
};

// sum_j q_j * x_j over 32 values for the low (A) and high (B) 4/5-bit fields held
// as bytes of lo[i]/hi[i] (value 4i+k in byte k).  Exact small integers are made
// with the 2^23 magic-number trick; f32x2 FMAs accumulate.
__device__ __forceinline__ void byte_field_dot(const uint32_t (&lo)[8], const uint32_t (&hi)[8],
                                               const ChunkX& x, float& sA, float& sB) {
  const float2 mg = make_float2(-kMagic, -kMagic);
  float2 a0 = make_float2(0.f, 0.f), a1 = a0, b0 = a0, b1 = a0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 l01 = __fadd2_rn(make_float2(byte_magic(lo[i], 0), byte_magic(lo[i], 1)), mg);
    const float2 l23 = __fadd2_rn(make_float2(byte_magic(lo[i], 2), byte_magic(lo[i], 3)), mg);
    const float2 h01 = __fadd2_rn(make_float2(byte_magic(hi[i], 0), byte_magic(hi[i], 1)), mg);
    const float2 h23 = __fadd2_rn(make_float2(byte_magic(hi[i], 2), byte_magic(hi[i], 3)), mg);
    a0 = __ffma2_rn(l01, x.a[2 * i], a0);
    a1 = __ffma2_rn(l23, x.a[2 * i + 1], a1);
    b0 = __ffma2_rn(h01, x.b[2 * i], b0);
    b1 = __ffma2_rn(h23, x.b[2 * i + 1], b1);
  }
  sA = (a0.x + a0.y) + (a1.x + a1.y);
  sB = (b0.x + b0.y) + (b1.x + b1.y);
}

// 32 packed Q4_K nibble bytes (two uint4) -> dot products of both nibble halves.
__device__ __forceinline__ void q4_nibble_dot(const uint4 q0, const uint4 q1, const ChunkX& x,
                                              float& sA, float& sB) {
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    lo[i] = w[i] & 0x0f0f0f0fu;
    hi[i] = (w[i] >> 4u) & 0x0f0f0f0fu;
  }
  byte_field_dot(lo, hi, x, sA, sB);
}

template <int FMT>
__device__ __forceinline__ float chunk_dot(const uint8_t* rp, const uint8_t* rm, uint32_t c,
                                           const ChunkX& x, const uint16_t* kgrid,
                                           const uint32_t* grid3);

// Q4_K raw block header: d, dmin, scales -> the chunk's two (scale, min) products.
__device__ __forceinline__ float q4k_header_combine(const uint4 h, uint32_t g, float sA, float sB,
                                                    const ChunkX& x) {
  const float d = h2f(h.x), dmin = h2f(h.x >> 16);
  uint32_t sc0, m0, sc1, m1;
  scale_min_k4(2u * g, h.y, h.z, h.w, sc0, m0);
  scale_min_k4(2u * g + 1u, h.y, h.z, h.w, sc1, m1);
  return d * (static_cast<float>(sc0) * sA + static_cast<float>(sc1) * sB) -
         dmin * (static_cast<float>(m0) * x.sa + static_cast<float>(m1) * x.sb);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q4K_RAW>(const uint8_t* rp, const uint8_t*,
                                                           uint32_t c, const ChunkX& x,
                                                           const uint16_t*, const uint32_t*) {
  const uint8_t* blk = rp + (c >> 2) * 144u;
  const uint32_t g = c & 3u;
  const uint4 h = *reinterpret_cast<const uint4*>(blk);
  const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 16u + 32u * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 32u + 32u * g);
  float sA, sB;
  q4_nibble_dot(q0, q1, x, sA, sB);
  return q4k_header_combine(h, g, sA, sB, x);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q4K_SPLIT_NATIVE>(
    const uint8_t* rp, const uint8_t* rm, uint32_t c, const ChunkX& x, const uint16_t*,
    const uint32_t*) {
  const uint32_t b = c >> 2, g = c & 3u;
  const uint4 h = *reinterpret_cast<const uint4*>(rm + b * 16u);
  const uint4 q0 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g + 16u);
  float sA, sB;
  q4_nibble_dot(q0, q1, x, sA, sB);
  return q4k_header_combine(h, g, sA, sB, x);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q4K_SPLIT_PREDECODED>(
    const uint8_t* rp, const uint8_t* rm, uint32_t c, const ChunkX& x, const uint16_t*,
    const uint32_t*) {
  const uint32_t b = c >> 2, g = c & 3u;
  const float4 sm = *reinterpret_cast<const float4*>(rm + b * 64u + 16u * g);
  const uint4 q0 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g + 16u);
  float sA, sB;
  q4_nibble_dot(q0, q1, x, sA, sB);
  return (sm.x * sA + sm.z * sB) - (sm.y * x.sa + sm.w * x.sb);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q4K_SPLIT_HALF>(
    const uint8_t* rp, const uint8_t* rm, uint32_t c, const ChunkX& x, const uint16_t*,
    const uint32_t*) {
  const uint32_t b = c >> 2, g = c & 3u;
  const uint2 hm = *reinterpret_cast<const uint2*>(rm + b * 32u + 8u * g);
  const uint4 q0 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g + 16u);
  float sA, sB;
  q4_nibble_dot(q0, q1, x, sA, sB);
  return (h2f(hm.x) * sA + h2f(hm.y) * sB) - (h2f(hm.x >> 16) * x.sa + h2f(hm.y >> 16) * x.sb);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q4K_SPLIT_COMPACT>(
    const uint8_t* rp, const uint8_t* rm, uint32_t c, const ChunkX& x, const uint16_t*,
    const uint32_t*) {
  const uint32_t b = c >> 2, g = c & 3u;
  const uint8_t* m = rm + b * 20u;
  const uint32_t dd = *reinterpret_cast<const uint32_t*>(m);
  const uint32_t sc = ld_u16(m + 4u + 2u * g);
  const uint32_t mn = ld_u16(m + 12u + 2u * g);
  const uint4 q0 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g + 16u);
  float sA, sB;
  q4_nibble_dot(q0, q1, x, sA, sB);
  return h2f(dd) * (static_cast<float>(sc & 0xffu) * sA + static_cast<float>(sc >> 8) * sB) -
         h2f(dd >> 16) * (static_cast<float>(mn & 0xffu) * x.sa + static_cast<float>(mn >> 8) * x.sb);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q5K>(const uint8_t* rp, const uint8_t*,
                                                       uint32_t c, const ChunkX& x,
                                                       const uint16_t*, const uint32_t*) {
  const uint8_t* blk = rp + (c >> 2) * 176u;
  const uint32_t g = c & 3u;
  const uint4 h = *reinterpret_cast<const uint4*>(blk);
  const uint4 qh0 = *reinterpret_cast<const uint4*>(blk + 16u);
  const uint4 qh1 = *reinterpret_cast<const uint4*>(blk + 32u);
  const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 48u + 32u * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 64u + 32u * g);
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  const uint32_t hw[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
  const uint32_t sl = 2u * g, sh = 2u * g + 1u;
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    lo[i] = (w[i] & 0x0f0f0f0fu) | (((hw[i] >> sl) & 0x01010101u) << 4u);
    hi[i] = ((w[i] >> 4u) & 0x0f0f0f0fu) | (((hw[i] >> sh) & 0x01010101u) << 4u);
  }
  float sA, sB;
  byte_field_dot(lo, hi, x, sA, sB);
  return q4k_header_combine(h, g, sA, sB, x);
}

// sum_l sign_l * (2 k_l + 1) * x_l for one IQ2_S group of 8 values: kgrid entry G
// (eight 2-bit k), sign byte S, x = four float2 (values 0..7).
__device__ __forceinline__ float iq2_group_dot(uint32_t G, uint32_t S, const float2* xs) {
  float2 acc = make_float2(0.f, 0.f);
  const float2 mg = make_float2(-kMagic, -kMagic);
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t l0 = 2u * p, l1 = 2u * p + 1u;
    const float m0 = __uint_as_float(0x4b000001u | (((G >> (2u * l0)) & 3u) << 1u));
    const float m1 = __uint_as_float(0x4b000001u | (((G >> (2u * l1)) & 3u) << 1u));
    const float2 m = __fadd2_rn(make_float2(m0, m1), mg);
    const float x0 = __uint_as_float(__float_as_uint(xs[p].x) ^ (((S >> l0) & 1u) << 31u));
    const float x1 = __uint_as_float(__float_as_uint(xs[p].y) ^ (((S >> l1) & 1u) << 31u));
    acc = __ffma2_rn(m, make_float2(x0, x1), acc);
  }
  return acc.x + acc.y;
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_IQ2S>(const uint8_t* rp, const uint8_t*,
                                                        uint32_t c, const ChunkX& x,
                                                        const uint16_t* kgrid, const uint32_t*) {
  const uint8_t* blk = rp + (c >> 2) * 82u;
  const uint32_t sub = c & 3u;
  const float d = h2f(ld_u16(blk));
  const uint32_t gl0 = ld_u32_a2(blk + 2u + 8u * sub), gl1 = ld_u32_a2(blk + 6u + 8u * sub);
  const uint32_t sg0 = ld_u32_a2(blk + 34u + 8u * sub), sg1 = ld_u32_a2(blk + 38u + 8u * sub);
  const uint32_t qh = ld_u16(blk + 66u + 2u * sub);
  const uint32_t sc = ld_u16(blk + 74u + 2u * sub);
  float res = 0.f;
#pragma unroll
  for (int ib = 0; ib < 2; ++ib) {
    const uint32_t gl = ib ? gl1 : gl0, sg = ib ? sg1 : sg0;
    const uint32_t qhb = (qh >> (8u * ib)) & 0xffu, sb = (sc >> (8u * ib)) & 0xffu;
    const float2* xs = ib ? x.b : x.a;
    float p[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint32_t idx = byte_of(gl, g) | ((qhb << (8u - 2u * g)) & 0x300u);
      p[g] = iq2_group_dot(kgrid[idx], byte_of(sg, g), xs + 4 * g);
    }
    const float s_lo = d * (0.5f + static_cast<float>(sb & 0x0fu)) * 0.25f;
    const float s_hi = d * (0.5f + static_cast<float>(sb >> 4u)) * 0.25f;
    res += s_lo * (p[0] + p[1]) + s_hi * (p[2] + p[3]);
  }
  return res;
}

// sum over 4 values of sign * magnitude * x for one IQ3_S grid entry (4 byte
// magnitudes), sign bits sbits (bit l for value l), x = two float2.
__device__ __forceinline__ float iq3_quad_dot(uint32_t grid, uint32_t sbits, const float2* xs) {
  const float2 mg = make_float2(-kMagic, -kMagic);
  const float2 m01 = __fadd2_rn(make_float2(byte_magic(grid, 0), byte_magic(grid, 1)), mg);
  const float2 m23 = __fadd2_rn(make_float2(byte_magic(grid, 2), byte_magic(grid, 3)), mg);
  const float x0 = __uint_as_float(__float_as_uint(xs[0].x) ^ ((sbits & 1u) << 31u));
  const float x1 = __uint_as_float(__float_as_uint(xs[0].y) ^ (((sbits >> 1u) & 1u) << 31u));
  const float x2 = __uint_as_float(__float_as_uint(xs[1].x) ^ (((sbits >> 2u) & 1u) << 31u));
  const float x3 = __uint_as_float(__float_as_uint(xs[1].y) ^ (((sbits >> 3u) & 1u) << 31u));
  float2 acc = __ffma2_rn(m01, make_float2(x0, x1), make_float2(0.f, 0.f));
  acc = __ffma2_rn(m23, make_float2(x2, x3), acc);
  return acc.x + acc.y;
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_IQ3S>(const uint8_t* rp, const uint8_t*,
                                                        uint32_t c, const ChunkX& x,
                                                        const uint16_t*, const uint32_t* grid3) {
  const uint8_t* blk = rp + (c >> 2) * 110u;
  const uint32_t sub = c & 3u;
  const float d = h2f(ld_u16(blk));
  uint32_t qs[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qs[i] = ld_u32_a2(blk + 2u + 16u * sub + 4u * i);
  const uint32_t qh = ld_u16(blk + 66u + 2u * sub);
  const uint32_t sg0 = ld_u32_a2(blk + 74u + 8u * sub), sg1 = ld_u32_a2(blk + 78u + 8u * sub);
  const uint32_t sb = blk[106u + sub];
  float res = 0.f;
#pragma unroll
  for (int ib = 0; ib < 2; ++ib) {
    const uint32_t qhb = (qh >> (8u * ib)) & 0xffu;
    const uint32_t sg = ib ? sg1 : sg0;
    const float2* xs = ib ? x.b : x.a;
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint32_t sbyte = byte_of(sg, g);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const uint32_t sel = 2u * g + p;  // byte index within this sub-block's 8 qs bytes
        const uint32_t qb = byte_of(qs[2 * ib + (sel >> 2)], sel & 3u);
        const uint32_t idx = qb | (((qhb >> (2u * g + p)) & 1u) << 8u);
        acc += iq3_quad_dot(grid3[idx], sbyte >> (4u * p), xs + 4 * g + 2 * p);
      }
    }
    const uint32_t nib = ib ? (sb >> 4u) : (sb & 0x0fu);
    res += d * static_cast<float>(1u + 2u * nib) * acc;
  }
  return res;
}

}  // namespace qg
