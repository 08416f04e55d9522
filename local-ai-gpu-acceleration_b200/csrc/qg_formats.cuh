// qg_formats.cuh -- per-format quant readers for the sm_100a decode kernels.
//
// Two readers per format:
//  * dequant_value<FMT>: one value, same arithmetic and order as the reference's
//    CPU decode (runtime/apps/mixed_sequence_benchmark_runner/main.cpp:1086-1259,
//    device twins decode_kernels.cu:1504-1728) with explicit _rn operations so
//    nvcc cannot contract them -- bit-identical fp32 output.
//  * chunk_dot<FMT>: the GEMV inner product of one 64-column chunk of one row,
//    reading the row's bytes from shared memory (see the GEMV section below).
//
// A 64-column chunk c of a row covers columns [64c, 64c+64): for the K-quants the
// low/high nibbles of qs[32*(c%4) .. +32) of block c/4, for the IQ formats the two
// 32-value sub-blocks 2*(c%4), 2*(c%4)+1 of block c/4.
#pragma once

#include "iq_grids.h"
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
// GEMV chunk readers (shared memory), integer dot products.
//
// x is held by each thread as two signed-byte planes per 32-column half:
//   x_j ~= s * (hi_j + lo_j / 256),  s = max|x| / 126 over the half,
// |error| <= s / 256 <= 3.2e-5 * ||x||_inf per element, i.e. <= 3.2e-5 *
// ||w_row||_1 * ||x||_inf per output -- 30x inside the 1e-3 parity bound.  Every
// format is decoded to small non-negative integers u (bytes) so one dp4a handles
// four weights per plane:
//   Q4_K/Q5_K  u = q (4/5-bit quant);   row sum = d*sc*sum(q x) - dmin*m*sum(x)
//   IQ2_S      u = v + 8  = 2k XOR (sign ? 7 : 9)       (v = +-(2k+1))
//   IQ3_S      u = v + 15 = g  XOR (sign ? 0x0F : 0x11) (v = +-g, g odd <= 15)
// the IQ biases are removed with per-16-column sums of the x planes.

struct XChunk {
  uint32_t ah[8], al[8];  // half A (columns 0..31): hi / lo planes, word i = columns 4i..4i+3
  uint32_t bh[8], bl[8];  // half B (columns 32..63)
  float sa, sb;           // plane scales of the halves
  float suma, sumb;       // exact fp32 sums of x over the halves
  int qh[4], ql[4];       // plane byte sums per 16-column quarter (IQ bias removal)
};

__device__ __forceinline__ void quantize_half(const float (&v)[32], uint32_t (&hi)[8],
                                              uint32_t (&lo)[8], float& s, float& sum,
                                              int& qh0, int& ql0, int& qh1, int& ql1) {
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) m = fmaxf(m, fabsf(v[j]));
  // Pairwise-tree sum, the order warp_prepare_chunk's butterfly produces.
  float p[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) p[j] = v[2 * j] + v[2 * j + 1];
#pragma unroll
  for (int len = 8; len >= 1; len >>= 1) {
#pragma unroll
    for (int j = 0; j < len; ++j) p[j] = p[2 * j] + p[2 * j + 1];
  }
  sum = p[0];
  s = m > 0.f ? m * (1.0f / 126.0f) : 1.0f;
  const float inv = 1.0f / s;
  // Round to nearest even with the 1.5 * 2^23 magic number: for |u| < 2^22 the low
  // mantissa bits of u + 1.5*2^23 hold round(u) as a two's-complement integer.
  constexpr float kRound = 12582912.0f;
  constexpr int kRoundBits = 0x4b400000;
  qh0 = ql0 = qh1 = ql1 = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int ia[4], ib[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float u = v[4 * i + k] * inv;
      const float ur = u + kRound;
      ia[k] = __float_as_int(ur) - kRoundBits;
      const float r = (u - (ur - kRound)) * 256.0f;
      ib[k] = min(max(__float_as_int(r + kRound) - kRoundBits, -127), 127);
    }
    hi[i] = __byte_perm(__byte_perm(ia[0], ia[1], 0x0040), __byte_perm(ia[2], ia[3], 0x0040), 0x5410);
    lo[i] = __byte_perm(__byte_perm(ib[0], ib[1], 0x0040), __byte_perm(ib[2], ib[3], 0x0040), 0x5410);
    const int sa = (ia[0] + ia[1]) + (ia[2] + ia[3]);
    const int sb = (ib[0] + ib[1]) + (ib[2] + ib[3]);
    if (i < 4) {
      qh0 += sa;
      ql0 += sb;
    } else {
      qh1 += sa;
      ql1 += sb;
    }
  }
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
  return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// dot of 4 unsigned bytes of a with 4 signed bytes of b, plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Exact int -> float for small magnitudes with full-rate ALU/FMA ops (no I2F):
// u < 2^23 via the 2^23 magic number.
__device__ __forceinline__ float u2f_small(uint32_t u) {
  return __uint_as_float(0x4b000000u | u) - 8388608.0f;
}

// s * (ih + il / 256): the two plane sums combined exactly as the integer 256 ih + il
// (below 2^28 for every reader: |ih| <= 32 * 240 * 127), one conversion (the
// conversion unit is otherwise idle; rounding 2^-24 relative), one multiply by s / 256
// (a per-thread constant).
__device__ __forceinline__ float planes_value(int ih, int il, float s) {
  return __int2float_rn(ih * 256 + il) * (s * 0.00390625f);
}

// sum(q x) over both halves for 8 words of byte quants: A = lo[], B = hi[].
__device__ __forceinline__ void quant_dot(const uint32_t (&lo)[8], const uint32_t (&hi)[8],
                                          const XChunk& x, float& sA, float& sB) {
  int ah0 = 0, al0 = 0, bh0 = 0, bl0 = 0, ah1 = 0, al1 = 0, bh1 = 0, bl1 = 0;
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    ah0 = dp4a(lo[i], x.ah[i], ah0);
    al0 = dp4a(lo[i], x.al[i], al0);
    bh0 = dp4a(hi[i], x.bh[i], bh0);
    bl0 = dp4a(hi[i], x.bl[i], bl0);
    ah1 = dp4a(lo[i + 1], x.ah[i + 1], ah1);
    al1 = dp4a(lo[i + 1], x.al[i + 1], al1);
    bh1 = dp4a(hi[i + 1], x.bh[i + 1], bh1);
    bl1 = dp4a(hi[i + 1], x.bl[i + 1], bl1);
  }
  sA = planes_value(ah0 + ah1, al0 + al1, x.sa);
  sB = planes_value(bh0 + bh1, bl0 + bl1, x.sb);
}

// Q4_K: low nibbles are w & 0x0F0F0F0F; the high nibbles stay in place
// (w & 0xF0F0F0F0 = 16 * q, unsigned bytes) and the 1/16 goes into the scale.
__device__ __forceinline__ void q4_nibble_dot(const uint4 q0, const uint4 q1, const XChunk& x,
                                              float& sA, float& sB) {
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  int ah0 = 0, al0 = 0, bh0 = 0, bl0 = 0, ah1 = 0, al1 = 0, bh1 = 0, bl1 = 0;
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const uint32_t l0 = w[i] & 0x0f0f0f0fu, h0 = w[i] & 0xf0f0f0f0u;
    const uint32_t l1 = w[i + 1] & 0x0f0f0f0fu, h1 = w[i + 1] & 0xf0f0f0f0u;
    ah0 = dp4a(l0, x.ah[i], ah0);
    al0 = dp4a(l0, x.al[i], al0);
    bh0 = dp4a_us(h0, x.bh[i], bh0);
    bl0 = dp4a_us(h0, x.bl[i], bl0);
    ah1 = dp4a(l1, x.ah[i + 1], ah1);
    al1 = dp4a(l1, x.al[i + 1], al1);
    bh1 = dp4a_us(h1, x.bh[i + 1], bh1);
    bl1 = dp4a_us(h1, x.bl[i + 1], bl1);
  }
  sA = planes_value(ah0 + ah1, al0 + al1, x.sa);
  sB = planes_value(bh0 + bh1, bl0 + bl1, x.sb * 0.0625f);
}

// Shared-memory codebook tables of the IQ kernels, replicated so that lookups from
// one warp spread over the 32 banks instead of colliding (random indices into a
// single copy cost ~3.5 wavefronts per warp-wide lookup):
//  * C3 = kIq3Copies copies of a 4-byte table (IQ3_S grid): word (e*C3 + lane % C3);
//    with 32 copies every lane owns a bank (conflict-free), with 16 lanes k and k+16
//    share one (at most a 2-way conflict);
//  * 16 copies of an 8-byte table (IQ3_S sign masks): entry (e*16 + k) sits in bank pair
//    k, one bank pair per lane of a half-warp -> conflict-free;
//  * C = kIq2Copies copies of the 8-byte IQ2_S grid (bytes 2k+1): copy r = k % C occupies
//    only the bank pairs r + C*i, so 16/C lanes of a half-warp compete for 16/C pairs.
// The pointers are already offset to this lane's copy, so a lookup is one multiply-add:
// kgrid2[C e], grid3[C3 e], sign3[16 e].
#ifndef QG_IQ2S_KGRID_COPIES
#define QG_IQ2S_KGRID_COPIES 8u
#endif
constexpr uint32_t kIq2Copies = QG_IQ2S_KGRID_COPIES;
static_assert(kIq2Copies == 4u || kIq2Copies == 8u || kIq2Copies == 16u,
              "IQ2_S grid copies: 4, 8 or 16");
constexpr uint32_t kIq2TableBytes = 2048u * kIq2Copies * 4u;

// Byte masks of all eight sign bits of a byte b (< 256), with no nibble masking: lo byte i
// = 0xFF where bit i is set, hi byte i = 0xFF where bit 4 + i is set.  b * 0x80402010
// puts bit 3 - i at bit 8i + 7 and b * 0x08040201 puts bit 7 - i there; each multiplier's
// four partial products of a byte cover disjoint bit ranges (4-11, 13-20, 22-29, 31-38
// and 0-7, 9-16, 18-25, 27-34), so there are no carries and the other bits land away
// from bit 7 of each byte; a byte-reversing sign-replicating prmt then gives the masks.
__device__ __forceinline__ void sign_masks8(uint32_t b, uint32_t& lo, uint32_t& hi) {
  asm("prmt.b32 %0, %1, 0, 0x89AB;" : "=r"(lo) : "r"(b * 0x80402010u));
  asm("prmt.b32 %0, %1, 0, 0x89AB;" : "=r"(hi) : "r"(b * 0x08040201u));
}
// Byte G of w, zero-extended (one prmt).
template <int G>
__device__ __forceinline__ uint32_t byte_at(uint32_t w) {
  uint32_t r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "n"(0x4440 | G));
  return r;
}
// Odd magnitudes m (bytes) are negated by m ^ 0xFE (= -m in two's complement), so a
// weight word with its signs applied is mags ^ (mask & 0xFEFEFEFE).
// Byte g of `lo` in byte 0 and byte g of `hi` (< 128) in byte 1, zero above: the 16-bit
// value lo_g + 256 hi_g in one prmt (the sign-replicating selector on hi's byte g, whose
// top bit is clear, yields the zero bytes).
template <int G>
__device__ __forceinline__ uint32_t pair_bytes(uint32_t lo, uint32_t hi) {
  constexpr uint32_t sel = G | ((4 + G) << 4) | ((8 | (4 + G)) << 8) | ((8 | (4 + G)) << 12);
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(lo), "r"(hi), "n"(sel));
  return r;
}
// The four 2-bit fields of a byte b, one per byte: byte g = (b >> 2g) & 3.  Fields 0, 2 and
// fields 1, 3 are moved by two multiplies whose partial products do not overlap.
__device__ __forceinline__ uint32_t spread2x4(uint32_t b) {
  const uint32_t e = (b & 0x33u) * 0x1001u;      // field 0 -> bits 0-1, field 2 -> 16-17
  const uint32_t o = (b & 0xCCu) * 0x40040u;     // field 1 -> bits 8-9, field 3 -> 24-25
  return (e & 0x00030003u) | (o & 0x03000300u);
}
// The four bits of a nibble n, one per byte: byte i = bit i of n (positions 7j + i of the
// four partial products are all distinct, so no carries).
__device__ __forceinline__ uint32_t spread1x4(uint32_t n) {
  return (n * 0x00204081u) & 0x01010101u;
}
#ifndef QG_IQ3S_GRID_COPIES
#define QG_IQ3S_GRID_COPIES 32u
#endif
constexpr uint32_t kIq3Copies = QG_IQ3S_GRID_COPIES;
static_assert(kIq3Copies == 16u || kIq3Copies == 32u, "IQ3_S grid copies: 16 or 32");
// IQ3_S sign masks: computed in registers (0; measured 2% faster on B200 than the
// table, whose 8-byte lookups add shared-memory wavefronts) or from a shared table (1).
#ifndef QG_IQ3S_TABLE_SIGNS
#define QG_IQ3S_TABLE_SIGNS 0
#endif
constexpr bool kIq3TableSigns = QG_IQ3S_TABLE_SIGNS != 0;
constexpr uint32_t kIq3SignByte = 2048u * kIq3Copies;  // byte offset of the IQ3_S sign table
constexpr uint32_t kIq3TableBytes = kIq3SignByte + (kIq3TableSigns ? 32768u : 0u);

struct IqTables {
  const uint2* kgrid2;    // IQ2_S: 1024 entries x C copies (slot C e + k%C), 8 bytes 2k+1
  const uint32_t* grid3;  // IQ3_S: 512 entries x C3 copies (slot C3 e + lane%C3), 4 magnitudes
  const uint2* sign3;     // IQ3_S: 256 entries x 16 copies (slot 16e + k), bytes (sign ? 0xFE : 0)
  uint32_t k;             // lane % 16
};

template <int FMT>
__device__ __forceinline__ float chunk_dot(const uint8_t* rp, const uint8_t* rm, uint32_t c,
                                           const XChunk& x, const IqTables& t);

// Q4_K 16-byte header {d, dmin, scales[12]} -> the chunk's row contribution.  Both
// (scale, min) pairs 2g, 2g+1 of get_scale_min_k4 are unpacked two bytes at a time.
__device__ __forceinline__ float q4k_header_combine(const uint4 h, uint32_t g, float sA, float sB,
                                                    const XChunk& x) {
  const float d = h2f(h.x), dmin = h2f(h.x >> 16);
  const uint32_t sh = 16u * (g & 1u);
  const uint32_t y16 = (h.y >> sh) & 0xffffu, z16 = (h.z >> sh) & 0xffffu, w16 = (h.w >> sh) & 0xffffu;
  uint32_t scp, mnp;
  if (g < 2u) {
    scp = y16 & 0x3f3fu;
    mnp = z16 & 0x3f3fu;
  } else {
    scp = (w16 & 0x0f0fu) | ((y16 & 0xc0c0u) >> 2);
    mnp = ((w16 >> 4) & 0x0f0fu) | ((z16 & 0xc0c0u) >> 2);
  }
  const float sc0 = u2f_small(scp & 0xffu), sc1 = u2f_small(scp >> 8);
  const float m0 = u2f_small(mnp & 0xffu), m1 = u2f_small(mnp >> 8);
  return d * (sc0 * sA + sc1 * sB) - dmin * (m0 * x.suma + m1 * x.sumb);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q4K_RAW>(const uint8_t* rp, const uint8_t*,
                                                           uint32_t c, const XChunk& x,
                                                           const IqTables&) {
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
    const uint8_t* rp, const uint8_t* rm, uint32_t c, const XChunk& x, const IqTables&) {
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
    const uint8_t* rp, const uint8_t* rm, uint32_t c, const XChunk& x, const IqTables&) {
  const uint32_t b = c >> 2, g = c & 3u;
  const float4 sm = *reinterpret_cast<const float4*>(rm + b * 64u + 16u * g);
  const uint4 q0 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g + 16u);
  float sA, sB;
  q4_nibble_dot(q0, q1, x, sA, sB);
  return (sm.x * sA + sm.z * sB) - (sm.y * x.suma + sm.w * x.sumb);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q4K_SPLIT_HALF>(
    const uint8_t* rp, const uint8_t* rm, uint32_t c, const XChunk& x, const IqTables&) {
  const uint32_t b = c >> 2, g = c & 3u;
  const uint2 hm = *reinterpret_cast<const uint2*>(rm + b * 32u + 8u * g);
  const uint4 q0 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g + 16u);
  float sA, sB;
  q4_nibble_dot(q0, q1, x, sA, sB);
  return (h2f(hm.x) * sA + h2f(hm.y) * sB) - (h2f(hm.x >> 16) * x.suma + h2f(hm.y >> 16) * x.sumb);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q4K_SPLIT_COMPACT>(
    const uint8_t* rp, const uint8_t* rm, uint32_t c, const XChunk& x, const IqTables&) {
  const uint32_t b = c >> 2, g = c & 3u;
  const uint8_t* m = rm + b * 20u;
  const uint32_t dd = *reinterpret_cast<const uint32_t*>(m);
  const uint32_t sc = ld_u16(m + 4u + 2u * g);
  const uint32_t mn = ld_u16(m + 12u + 2u * g);
  const uint4 q0 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(rp + b * 128u + 32u * g + 16u);
  float sA, sB;
  q4_nibble_dot(q0, q1, x, sA, sB);
  return h2f(dd) * (u2f_small(sc & 0xffu) * sA + u2f_small(sc >> 8) * sB) -
         h2f(dd >> 16) * (u2f_small(mn & 0xffu) * x.suma + u2f_small(mn >> 8) * x.sumb);
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_Q5K>(const uint8_t* rp, const uint8_t*,
                                                       uint32_t c, const XChunk& x,
                                                       const IqTables&) {
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
  quant_dot(lo, hi, x, sA, sB);
  return q4k_header_combine(h, g, sA, sB, x);
}

// One IQ2_S sub-block (32 weights, 4 groups of 8) against one half of x: the integer
// sums of the two scale quarters (groups 0-1 with the low scale nibble, 2-3 with the
// high), scaled by (2 nib + 1), into (h, l) for the x planes.
__device__ __forceinline__ void iq2s_sub(uint32_t gl, uint32_t sg, uint32_t qhb, uint32_t scb,
                                         const uint32_t* H, const uint32_t* L,
                                         const IqTables& t, int& h, int& l) {
  const uint32_t h4 = spread2x4(qhb);
  uint32_t idx[4];
  idx[0] = pair_bytes<0>(gl, h4);
  idx[1] = pair_bytes<1>(gl, h4);
  idx[2] = pair_bytes<2>(gl, h4);
  idx[3] = pair_bytes<3>(gl, h4);
  int ih[2] = {0, 0}, il[2] = {0, 0};
  const uint32_t sbs[4] = {byte_at<0>(sg), byte_at<1>(sg), byte_at<2>(sg), byte_at<3>(sg)};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint2 k2 = t.kgrid2[idx[g] * kIq2Copies];
    uint32_t m0, m1;
    sign_masks8(sbs[g], m0, m1);
    const uint32_t v0 = k2.x ^ (m0 & 0xFEFEFEFEu);
    const uint32_t v1 = k2.y ^ (m1 & 0xFEFEFEFEu);
    ih[g >> 1] = dp4a(v1, H[2 * g + 1], dp4a(v0, H[2 * g], ih[g >> 1]));
    il[g >> 1] = dp4a(v1, L[2 * g + 1], dp4a(v0, L[2 * g], il[g >> 1]));
  }
  const int s0 = static_cast<int>(2u * (scb & 0x0fu) + 1u), s1 = static_cast<int>(2u * ((scb >> 4) & 0x0fu) + 1u);
  h = s0 * ih[0] + s1 * ih[1];
  l = s0 * il[0] + s1 * il[1];
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_IQ2S>(const uint8_t* rp, const uint8_t*,
                                                        uint32_t c, const XChunk& x,
                                                        const IqTables& t) {
  const uint8_t* blk = rp + (c >> 2) * 82u;
  const uint32_t sub = c & 3u;
  const float d = h2f(ld_u16(blk));
  const uint32_t gl0 = ld_u32_a2(blk + 2u + 8u * sub), gl1 = ld_u32_a2(blk + 6u + 8u * sub);
  const uint32_t sg0 = ld_u32_a2(blk + 34u + 8u * sub), sg1 = ld_u32_a2(blk + 38u + 8u * sub);
  const uint32_t qh = ld_u16(blk + 66u + 2u * sub);
  const uint32_t sc = ld_u16(blk + 74u + 2u * sub);
  int ha, la, hb, lb;
  iq2s_sub(gl0, sg0, qh & 0xffu, sc & 0xffu, x.ah, x.al, t, ha, la);
  iq2s_sub(gl1, sg1, qh >> 8, sc >> 8, x.bh, x.bl, t, hb, lb);
  // w = d (2 nib + 1) / 8 * v
  return (d * 0.125f) * (planes_value(ha, la, x.sa) + planes_value(hb, lb, x.sb));
}

// One IQ3_S sub-block (32 weights: 4 groups of two 4-weight grid entries) against one
// half of x: integer sums (h, l).
__device__ __forceinline__ void iq3s_sub(uint32_t q0, uint32_t q1, uint32_t qhb, uint32_t sg,
                                         const uint32_t* H, const uint32_t* L,
                                         const IqTables& t, int& h, int& l) {
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
  int ih = 0, il = 0;
  const uint32_t sbs[4] = {byte_at<0>(sg), byte_at<1>(sg), byte_at<2>(sg), byte_at<3>(sg)};
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t m0, m1;
    if constexpr (kIq3TableSigns) {
      const uint2 sm = t.sign3[sbs[g] << 4];
      m0 = sm.x;
      m1 = sm.y;
    } else {
      sign_masks8(sbs[g], m0, m1);
      m0 &= 0xFEFEFEFEu;
      m1 &= 0xFEFEFEFEu;
    }
    const uint32_t v0 = t.grid3[idx[2 * g] * kIq3Copies] ^ m0;
    const uint32_t v1 = t.grid3[idx[2 * g + 1] * kIq3Copies] ^ m1;
    ih = dp4a(v1, H[2 * g + 1], dp4a(v0, H[2 * g], ih));
    il = dp4a(v1, L[2 * g + 1], dp4a(v0, L[2 * g], il));
  }
  h = ih;
  l = il;
}

template <>
__device__ __forceinline__ float chunk_dot<QG_FMT_IQ3S>(const uint8_t* rp, const uint8_t*,
                                                        uint32_t c, const XChunk& x,
                                                        const IqTables& t) {
  const uint8_t* blk = rp + (c >> 2) * 110u;
  const uint32_t sub = c & 3u;
  const float d = h2f(ld_u16(blk));
  uint32_t qs[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qs[i] = ld_u32_a2(blk + 2u + 16u * sub + 4u * i);
  const uint32_t qh = ld_u16(blk + 66u + 2u * sub);
  const uint32_t sg0 = ld_u32_a2(blk + 74u + 8u * sub), sg1 = ld_u32_a2(blk + 78u + 8u * sub);
  const uint32_t sb = blk[106u + sub];
  int ha, la, hb, lb;
  iq3s_sub(qs[0], qs[1], qh & 0xffu, sg0, x.ah, x.al, t, ha, la);
  iq3s_sub(qs[2], qs[3], qh >> 8, sg1, x.bh, x.bl, t, hb, lb);
  // w = d (1 + 2 nib) * v, one scale per 32-weight sub-block (= one half of x)
  const float s0 = u2f_small(1u + 2u * (sb & 0x0fu)), s1 = u2f_small(1u + 2u * (sb >> 4));
  return d * (s0 * planes_value(ha, la, x.sa) + s1 * planes_value(hb, lb, x.sb));
}

// The replicated tables, built at compile time from the codebooks (in the IqTables
// layout: kIq2TableBytes for IQ2_S, kIq3TableBytes for IQ3_S) and copied into each
// CTA's shared memory with one bulk copy.
struct __align__(16) ReplicatedTables {
  uint32_t w[(kIq2TableBytes > kIq3TableBytes ? kIq2TableBytes : kIq3TableBytes) / 4u];
};

namespace tables_detail {
constexpr uint16_t kIq2Kgrid[1024] = {QG_IQ2S_KGRID_VALUES};
constexpr uint32_t kIq3Grid[512] = {QG_IQ3S_GRID_VALUES};

constexpr void put_sign_copies(ReplicatedTables& t, uint32_t word_base, uint32_t mag) {
  for (uint32_t e = 0; e < 256u; ++e) {
    uint32_t lo = 0u, hi = 0u;
    for (uint32_t l = 0; l < 4u; ++l) {
      lo |= (((e >> l) & 1u) ? mag : 0u) << (8u * l);
      hi |= (((e >> (l + 4u)) & 1u) ? mag : 0u) << (8u * l);
    }
    for (uint32_t r = 0; r < 16u; ++r) {
      t.w[word_base + 2u * ((e << 4) | r)] = lo;
      t.w[word_base + 2u * ((e << 4) | r) + 1u] = hi;
    }
  }
}

constexpr ReplicatedTables make_iq2s() {
  ReplicatedTables t{};
  for (uint32_t e = 0; e < 1024u; ++e) {
    const uint32_t G = kIq2Kgrid[e];
    uint32_t lo = 0u, hi = 0u;
    for (uint32_t l = 0; l < 4u; ++l) {
      lo |= ((((G >> (2u * l)) & 3u) << 1) | 1u) << (8u * l);
      hi |= ((((G >> (2u * (l + 4u))) & 3u) << 1) | 1u) << (8u * l);
    }
    for (uint32_t r = 0; r < kIq2Copies; ++r) {
      const uint32_t slot = kIq2Copies * e + r;
      t.w[2u * slot] = lo;
      t.w[2u * slot + 1u] = hi;
    }
  }
  return t;
}

constexpr ReplicatedTables make_iq3s() {
  ReplicatedTables t{};
  for (uint32_t e = 0; e < 512u; ++e) {
    for (uint32_t r = 0; r < kIq3Copies; ++r) t.w[e * kIq3Copies + r] = kIq3Grid[e];
  }
  if (kIq3TableSigns) put_sign_copies(t, kIq3SignByte / 4u, 0xfeu);
  return t;
}
}  // namespace tables_detail

extern __device__ const ReplicatedTables g_iq2s_tables;
extern __device__ const ReplicatedTables g_iq3s_tables;

template <int FMT>
__device__ __forceinline__ const ReplicatedTables* replicated_tables() {
  return FMT == QG_FMT_IQ2S ? &g_iq2s_tables : &g_iq3s_tables;
}

// All-thread copy of the format's tables into shared memory (fallback kernels).
template <int FMT>
__device__ __forceinline__ void build_iq_tables(uint8_t* base, uint32_t tid, uint32_t n) {
  if (FMT == QG_FMT_IQ2S || FMT == QG_FMT_IQ3S) {
    const uint4* src = reinterpret_cast<const uint4*>(replicated_tables<FMT>());
    uint4* dst = reinterpret_cast<uint4*>(base);
    constexpr uint32_t kVecs = (FMT == QG_FMT_IQ2S ? kIq2TableBytes : kIq3TableBytes) / 16u;
    for (uint32_t i = tid; i < kVecs; i += n) dst[i] = __ldg(src + i);
  }
}

template <int FMT>
__device__ __forceinline__ IqTables iq_tables(const uint8_t* base, uint32_t lane) {
  IqTables t{};
  t.k = lane & 15u;
  if (FMT == QG_FMT_IQ2S) {
    t.kgrid2 = reinterpret_cast<const uint2*>(base) + (t.k & (kIq2Copies - 1u));
  } else if (FMT == QG_FMT_IQ3S) {
    t.grid3 = reinterpret_cast<const uint32_t*>(base) + (lane & (kIq3Copies - 1u));
    t.sign3 = reinterpret_cast<const uint2*>(base + kIq3SignByte) + t.k;
  }
  return t;
}

constexpr uint32_t iq_table_bytes(int fmt) {
  return fmt == QG_FMT_IQ2S ? kIq2TableBytes : fmt == QG_FMT_IQ3S ? kIq3TableBytes : 0u;
}

// A prepared activation: x quantized once (qg_act_prepare) into one 176-byte record
// per 64-column chunk, the XChunk a GEMV thread would otherwise compute itself.
struct __align__(16) ActChunk {
  uint32_t ah[8], al[8], bh[8], bl[8];
  float sa, sb, suma, sumb;
  int qh[4], ql[4];
};
static_assert(sizeof(ActChunk) == 176, "prepared activation record is 176 bytes");

__device__ __forceinline__ void load_act_chunk(const ActChunk* __restrict__ src, XChunk& x) {
  const uint4* p = reinterpret_cast<const uint4*>(src);
  uint4 v[11];
#pragma unroll
  for (int i = 0; i < 11; ++i) v[i] = __ldg(p + i);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    x.ah[4 * i] = v[i].x; x.ah[4 * i + 1] = v[i].y; x.ah[4 * i + 2] = v[i].z; x.ah[4 * i + 3] = v[i].w;
    x.al[4 * i] = v[2 + i].x; x.al[4 * i + 1] = v[2 + i].y; x.al[4 * i + 2] = v[2 + i].z; x.al[4 * i + 3] = v[2 + i].w;
    x.bh[4 * i] = v[4 + i].x; x.bh[4 * i + 1] = v[4 + i].y; x.bh[4 * i + 2] = v[4 + i].z; x.bh[4 * i + 3] = v[4 + i].w;
    x.bl[4 * i] = v[6 + i].x; x.bl[4 * i + 1] = v[6 + i].y; x.bl[4 * i + 2] = v[6 + i].z; x.bl[4 * i + 3] = v[6 + i].w;
  }
  x.sa = __uint_as_float(v[8].x); x.sb = __uint_as_float(v[8].y);
  x.suma = __uint_as_float(v[8].z); x.sumb = __uint_as_float(v[8].w);
  x.qh[0] = v[9].x; x.qh[1] = v[9].y; x.qh[2] = v[9].z; x.qh[3] = v[9].w;
  x.ql[0] = v[10].x; x.ql[1] = v[10].y; x.ql[2] = v[10].z; x.ql[3] = v[10].w;
}

__device__ __forceinline__ void store_act_chunk(const XChunk& x, ActChunk* dst) {
  uint4* p = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    p[i] = make_uint4(x.ah[4 * i], x.ah[4 * i + 1], x.ah[4 * i + 2], x.ah[4 * i + 3]);
    p[2 + i] = make_uint4(x.al[4 * i], x.al[4 * i + 1], x.al[4 * i + 2], x.al[4 * i + 3]);
    p[4 + i] = make_uint4(x.bh[4 * i], x.bh[4 * i + 1], x.bh[4 * i + 2], x.bh[4 * i + 3]);
    p[6 + i] = make_uint4(x.bl[4 * i], x.bl[4 * i + 1], x.bl[4 * i + 2], x.bl[4 * i + 3]);
  }
  p[8] = make_uint4(__float_as_uint(x.sa), __float_as_uint(x.sb), __float_as_uint(x.suma),
                    __float_as_uint(x.sumb));
  p[9] = make_uint4(x.qh[0], x.qh[1], x.qh[2], x.qh[3]);
  p[10] = make_uint4(x.ql[0], x.ql[1], x.ql[2], x.ql[3]);
}

// One warp quantizes one 64-column chunk into its ActChunk: lane l holds columns 2l,
// 2l+1 (half A = lanes 0-15, half B = lanes 16-31).  Same arithmetic as quantize_half
// (scale = max|x| / 126 per half, magic-number rounding), so a chunk prepared here is
// bit-identical to one quantized inside the GEMV.
__device__ __forceinline__ void warp_prepare_chunk(float v0, float v1, ActChunk* dst) {
  const uint32_t lane = threadIdx.x & 31u;
  float m = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  const float s = m > 0.f ? m * (1.0f / 126.0f) : 1.0f;
  const float inv = 1.0f / s;
  constexpr float kRound = 12582912.0f;
  constexpr int kRoundBits = 0x4b400000;
  int ia[2], ib[2];
  const float v[2] = {v0, v1};
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float u = v[k] * inv;
    const float ur = u + kRound;
    ia[k] = __float_as_int(ur) - kRoundBits;
    const float r = (u - (ur - kRound)) * 256.0f;
    ib[k] = min(max(__float_as_int(r + kRound) - kRoundBits, -127), 127);
  }
  // bytes of columns 2l, 2l+1; the even lane of a pair assembles the 4-column word
  const uint32_t h2 = __byte_perm(ia[0], ia[1], 0x0040), l2 = __byte_perm(ib[0], ib[1], 0x0040);
  const uint32_t hn = __shfl_down_sync(0xffffffffu, h2, 1), ln = __shfl_down_sync(0xffffffffu, l2, 1);
  // sums: exact fp32 over the half (tree order), plane sums over 16-column quarters
  float t = v0 + v1;
  int qh = ia[0] + ia[1], ql = ib[0] + ib[1];
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) {
    t += __shfl_xor_sync(0xffffffffu, t, off);
    qh += __shfl_xor_sync(0xffffffffu, qh, off);
    ql += __shfl_xor_sync(0xffffffffu, ql, off);
  }
  t += __shfl_xor_sync(0xffffffffu, t, 8);
  const uint32_t half = lane >> 4, word = (lane & 15u) >> 1;
  uint32_t* w = reinterpret_cast<uint32_t*>(dst);
  if ((lane & 1u) == 0u) {
    w[half * 16u + word] = __byte_perm(h2, hn, 0x5410);
    w[half * 16u + 8u + word] = __byte_perm(l2, ln, 0x5410);
  }
  if ((lane & 15u) == 0u) {
    reinterpret_cast<float*>(w)[32u + half] = s;
    reinterpret_cast<float*>(w)[34u + half] = t;
  }
  if ((lane & 7u) == 0u) {
    w[36u + (lane >> 3)] = static_cast<uint32_t>(qh);
    w[40u + (lane >> 3)] = static_cast<uint32_t>(ql);
  }
}

// This thread's 64 columns of x, quantized to the two byte planes.
__device__ __forceinline__ void load_x_chunk(const float* __restrict__ xp, bool vec, XChunk& x) {
  float va[32], vb[32];
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(xp);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 a = __ldg(x4 + i), b = __ldg(x4 + 8 + i);
      va[4 * i] = a.x; va[4 * i + 1] = a.y; va[4 * i + 2] = a.z; va[4 * i + 3] = a.w;
      vb[4 * i] = b.x; vb[4 * i + 1] = b.y; vb[4 * i + 2] = b.z; vb[4 * i + 3] = b.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      va[i] = __ldg(xp + i);
      vb[i] = __ldg(xp + 32 + i);
    }
  }
  quantize_half(va, x.ah, x.al, x.sa, x.suma, x.qh[0], x.ql[0], x.qh[1], x.ql[1]);
  quantize_half(vb, x.bh, x.bl, x.sb, x.sumb, x.qh[2], x.ql[2], x.qh[3], x.ql[3]);
}

}  // namespace qg
