// qg_gemm_tc.cu -- batched dequantize-and-GEMM on the 5th-generation tensor cores
// (tcgen05.mma, operands and accumulators in tensor memory).  No reference counterpart:
// every reference matvec kernel is batch 1 (runtime/kernels/decode/decode_kernels.cu).
//
//   Y[b, r] = sum_c W[r, c] * X[b, c]     b < batch <= 32, W a resident GGUF pack
//
// Numerics.  Every supported format's weight is a per-block fp32 scale times a small
// integer, and that integer is exact in fp16:
//   Q4_K   w = d*(sc*q) - dmin*m           sc*q <= 945, m <= 63
//   Q5_K   w = d*(sc*q) - dmin*m           sc*q <= 1953
//   IQ2_S  w = (d/8) * (2s+1)(2k+1) sign   |int| <= 217
//   IQ3_S  w = d * (1+2s) g sign           |int| <= 465
// x is held in fp16 as xh = x * 2^-e, one power of two per batch row with
// max|xh| <= 1024.  Per block the tensor core forms
//   accq[r, b] = sum_c int(r, c) * xh(b, c)
//   accm[r, b] = sum_j m(r, j) * (sum of xh(b, c) over 32-column sub-block j)
// (the sub-block sums carried as an fp16 hi + lo pair), the epilogue accumulates
//   d * accq - dmin * accm
// in fp32 and scales the row result by 2^e.  The result is sum_c w(r, c) * x~(b, c)
// with x~ the fp16-rounded x, so |error| <= 2^-11 * ||w_row||_1 * ||x_b||_inf plus
// fp32 accumulation -- half the reference's 1e-3 parity bound.
//
// Work.  The (128-row tile, 256-column block) units of the matrix are split into one
// contiguous range per CTA (stream-K), one CTA per SM, so every SM streams the same
// number of weight bytes.  A tile whose block range is split between CTAs is summed
// by whichever CTA finishes it last (per-row atomic counters, partial sums added in
// CTA order, so results are deterministic); no CTA ever waits for another.
//
// Data path of one unit.  The raw blocks of the tile's 128 rows land in shared memory
// (one 2-D tensor copy); each dequantize thread owns one row and one half of the block
// and writes its 128 fp16 integers straight into tensor memory (tcgen05.st, row = TMEM
// lane), where the MMA reads them as the A operand; only x (the B operand) and the
// small K-quant min tile are read from shared memory.  Tensor memory (512 columns): 4
// accumulator slots of 2*NB columns (q and min parts) at columns [0, 8 NB), then A
// slots of 128 columns up to column 512 (3 for N=16, 2 for N=32).
//
// CTA roles (15 warps, one CTA per SM):
//   warp 0      weight producer: one 2-D tensor copy per unit (cp.async.bulk.tensor, a
//               box of 128 rows x one block, plain form) into a raw ring -- or, when
//               the row stride is not a 16-B multiple, one 1-D bulk copy per row;
//   warp 1      allocates tensor memory; lane 0 issues the MMAs (M=128, N=16|32, K=16);
//   warps 2-9   dequantize: warp w handles rows 32*(w%4).. (its tensor-memory lanes)
//               and half (w-2)/4 of every block;
//   warps 10-13 epilogue: tcgen05.ld of the block accumulators, fp32 block scales,
//               row results or partial sums to global memory;
//   warp 14     x producer: one 1-D bulk copy of the prepared x block per unit.
// Every mbarrier wait is bounded (QG_ERR_WAIT_TIMEOUT in the error word, then all
// roles stop, in-flight copies and MMAs are drained and tensor memory is freed).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

#include "qg_formats.cuh"
#include "qg_host.h"

namespace qg {
namespace {

constexpr uint32_t kTileM = 128;
// Batch from which qg_gemm_batched uses the tensor cores, set by measurement on B200
// (Q4_K 28672x8192): the CUDA-core multi-vector GEMV takes 48.6 / 77 / 114 us at batch
// 2 / 4 / 8, these tiles 80 / 80 / 79 us -- the 8-vector GEMV is bound by the half-rate
// integer dot-product pipe (4 dp2a per weight).
constexpr uint32_t kTcMinBatch = 5;
constexpr uint32_t kBlockCols = 256;
constexpr uint32_t kA2Bytes = kTileM * 16u * 2u;  // min tile: 128 rows x K=16 fp16
constexpr uint32_t kXStages = 4;
constexpr uint32_t kAccSlots = 4;
constexpr uint32_t kTmemCols = 512;
// first tensor-memory column of the A slots, and their number
template <uint32_t NB>
__host__ __device__ constexpr uint32_t tmem_a() { return kAccSlots * 2u * NB; }
template <uint32_t NB>
__host__ __device__ constexpr uint32_t a_slots() { return (kTmemCols - tmem_a<NB>()) / 128u; }
constexpr uint32_t kWarps = 15;
constexpr uint32_t kThreads = kWarps * 32u;
constexpr uint32_t kDequantWarp0 = 2, kEpilogueWarp0 = 10, kXWarp = 14;
constexpr uint32_t kSmemLimit = 232448;  // 227 KB: the opt-in maximum per block
constexpr uint32_t kMaxRawStages = 8;
constexpr uint32_t kMaxTcPolls = 4000;   // bounded waits: suspended polls of up to kPollNs
constexpr uint32_t kMaxSpinPolls = 1u << 26;  // bounded spin of the MMA thread (~1 s)
constexpr uint32_t kPollNs = 500000;

template <int FMT>
struct TcFmt;
template <>
struct TcFmt<QG_FMT_Q4K_RAW> {
  static constexpr uint32_t bpb = 144, rowb = 144, table_bytes = 0;
  static constexpr bool has_min = true, window = false;
};
template <>
struct TcFmt<QG_FMT_Q5K> {
  static constexpr uint32_t bpb = 176, rowb = 176, table_bytes = 0;
  static constexpr bool has_min = true, window = false;
};
// IQ blocks are not 16-B multiples: each row's block is fetched as the 16-B aligned
// window around it (<= 96 / 128 bytes); slots are padded so the 32 rows a warp reads
// start in distinct 16-B bank groups.
template <>
struct TcFmt<QG_FMT_IQ2S> {
  static constexpr uint32_t bpb = 82, rowb = 112, table_bytes = 16384 + 4096;
  static constexpr bool has_min = false, window = true;
};
template <>
struct TcFmt<QG_FMT_IQ3S> {
  static constexpr uint32_t bpb = 110, rowb = 144, table_bytes = 4096 + 4096;
  static constexpr bool has_min = false, window = true;
};

template <int FMT, uint32_t NB>
struct TcLayout {
  using F = TcFmt<FMT>;
  static constexpr uint32_t xrec = NB * 544u;  // fp16 x tile (NB x 256) + sub-block sums (NB x 16)
  static constexpr uint32_t a2_off = 0;
  static constexpr uint32_t a_slots = qg::a_slots<NB>();
  static constexpr uint32_t x_off = a2_off + (F::has_min ? a_slots * kA2Bytes : 0u);
  static constexpr uint32_t t_off = x_off + kXStages * xrec;
  static constexpr uint32_t raw_off = (t_off + F::table_bytes + 1023u) & ~1023u;
  static constexpr uint32_t raw_stage = kTileM * F::rowb;
  // barriers, tensor-memory address, flags (512 B), then the block scales of the
  // accumulator slots' units: [kAccSlots][2][128] fp32 (d-scale, dmin per row)
  static constexpr uint32_t scl_rel = 512;
  static constexpr uint32_t misc = scl_rel + kAccSlots * 2u * kTileM * 4u;
  static constexpr uint32_t slack = 1024;
  static constexpr uint32_t raw_stages_fit = (kSmemLimit - raw_off - misc - slack) / raw_stage;
  static constexpr uint32_t raw_stages = raw_stages_fit > kMaxRawStages ? kMaxRawStages : raw_stages_fit;
  static_assert(raw_stages >= 3u, "shared memory budget");
  static constexpr uint32_t bar_off = raw_off + raw_stages * raw_stage;
  static constexpr uint32_t smem = bar_off + misc + slack;
  static_assert(a_slots >= 2u, "tensor-memory layout");
};

// ---------------------------------------------------------------------------
// tcgen05 / UMMA primitives (PTX ISA 8.7, sm_100a).

// Shared-memory matrix descriptor, K-major without swizzle: core matrices of 8 rows x
// 16 bytes stored contiguously; the two core matrices along K (one K=16 step) are
// 128 B apart (leading byte offset), consecutive 8-row groups 256 B apart (stride
// byte offset); descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128u >> 4) << 16) |
         (static_cast<uint64_t>(256u >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor, kind::f16: fp16 A and B (K-major), fp32 D, M=128, N=NB.
template <uint32_t NB>
__host__ __device__ constexpr uint32_t umma_idesc() {
  return (1u << 4) | ((NB >> 3) << 17) | ((kTileM >> 4) << 24);
}

// D (tensor memory) (+)= A (shared-memory descriptor) x B (shared-memory descriptor).
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// D (tensor memory) (+)= A (tensor memory: row m = lane m, fp16 element k in column
// k/2) x B (shared-memory descriptor).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp gets its lane's 16.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Thread i of the warp writes 16 consecutive 32-bit columns of its lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&w)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]), "r"(w[8]),
      "r"(w[9]), "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]), "r"(w[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 2-D tiled tensor copy global -> shared of the box at (x, y) of `tmap` (a kernel
// parameter), completing on `bar`; plain form, the source is this GPU's memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tmap, int32_t x, int32_t y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// try_wait that suspends the thread (up to kPollNs) until the phase completes, so
// waiting warps do not take issue slots from the working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kPollNs)
      : "memory");
  return ok != 0u;
}

// Bounded wait of at most kMaxTcPolls suspended polls; gives up early once another
// role has set the CTA's abort flag.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
  for (uint32_t it = 0; it < kMaxTcPolls; ++it) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (*abort != 0u) return false;
  }
  atomicOr(&g_error_word, QG_ERR_WAIT_TIMEOUT);
  *abort = 1u;
  return false;
}

// Spinning variant for the MMA-issuing thread, the pipeline's critical path: a
// non-blocking poll of a completed phase costs a few cycles where a suspending one can
// cost hundreds under load (measured on B200: Q4_K 28672x8192 at batch 16 takes 79.5 us
// with this spin, 88 us with suspending try_waits).  Up to three phases at once (b1 may
// be null): the polls are independent, so their latencies overlap.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0u;
}

__device__ __forceinline__ bool tc_spin3(uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2, uint64_t* b3,
                                         uint32_t p3, volatile uint32_t* abort) {
  bool ok1 = b1 == nullptr, ok2 = false, ok3 = false;
  for (uint32_t it = 0; it < kMaxSpinPolls; ++it) {
    const bool r1 = ok1 || mbar_test_wait(b1, p1);
    const bool r2 = ok2 || mbar_test_wait(b2, p2);
    const bool r3 = ok3 || mbar_test_wait(b3, p3);
    ok1 = r1;
    ok2 = r2;
    ok3 = r3;
    if (ok1 && ok2 && ok3) return true;
    if ((it & 1023u) == 1023u && *abort != 0u) return false;
  }
  atomicOr(&g_error_word, QG_ERR_WAIT_TIMEOUT);
  *abort = 1u;
  return false;
}

// Warp-wide tc_wait: lane 0 waits, the warp learns the outcome.
__device__ __forceinline__ bool tc_wait_warp(uint64_t* bar, uint32_t parity, volatile uint32_t* abort,
                                             uint32_t lane) {
  uint32_t ok = 0;
  if (lane == 0u) ok = tc_wait(bar, parity, abort) ? 1u : 0u;
  return __shfl_sync(0xffffffffu, ok, 0) != 0u;
}

// ---------------------------------------------------------------------------
// Shared-memory layout of the x tile (UMMA canonical K-major, no swizzle): byte offset
// of element (b, c) of one block (16 K-steps of NB rows x 16 columns).
template <uint32_t NB>
__device__ __forceinline__ uint32_t x_elem(uint32_t b, uint32_t c) {
  return (c >> 4) * (NB * 32u) + (b >> 3) * 256u + ((c >> 3) & 1u) * 128u + (b & 7u) * 16u +
         (c & 7u) * 2u;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// (1024 + q) as fp16 pairs from two bytes' low nibbles / (1024 + 16q) from the high
// nibbles; fma with (s, -1024 s) or (s/16, -64 s) then gives s*q exactly.
__device__ __forceinline__ uint32_t nib_lo(uint32_t pair) { return (pair & 0x000F000Fu) | 0x64006400u; }
__device__ __forceinline__ uint32_t nib_hi(uint32_t pair) { return (pair & 0x00F000F0u) | 0x64006400u; }
__device__ __forceinline__ uint32_t hfma_bits(uint32_t h, __half2 s, __half2 c) {
  return h2_bits(__hfma2(bits_h2(h), s, c));
}

// ---------------------------------------------------------------------------
// Per-format dequantization of one row's half block (128 columns).  The 128 fp16
// integers leave as 4 groups of 32 consecutive columns (16 words, fp16 pairs with the
// lower column in the low half): emit(g, words) for g = 0..3.

// min tile row r: K slots 0..7 and 8..15 both hold m[0..7] (against the hi and lo
// halves of the sub-block sums); canonical K-major layout like the x tile.
__device__ __forceinline__ void store_mins(uint32_t s0, uint32_t s1, uint32_t s2, uint32_t r, uint8_t* A2) {
  uint32_t m[8];
#pragma unroll
  for (uint32_t j = 0; j < 8u; ++j) {
    uint32_t sc;
    scale_min_k4(j, s0, s1, s2, sc, m[j]);
  }
  uint4 mm;
  mm.x = h2_bits(__floats2half2_rn(static_cast<float>(m[0]), static_cast<float>(m[1])));
  mm.y = h2_bits(__floats2half2_rn(static_cast<float>(m[2]), static_cast<float>(m[3])));
  mm.z = h2_bits(__floats2half2_rn(static_cast<float>(m[4]), static_cast<float>(m[5])));
  mm.w = h2_bits(__floats2half2_rn(static_cast<float>(m[6]), static_cast<float>(m[7])));
  const uint32_t o = (r >> 3) * 256u + (r & 7u) * 16u;
  *reinterpret_cast<uint4*>(A2 + o) = mm;
  *reinterpret_cast<uint4*>(A2 + o + 128u) = mm;
}

template <int FMT>
struct Dequant;

// Q4_K: block = d, dmin, scales[12], qs[128]; group g (64 columns) holds columns
// 64g + j (low nibble of qs[32g + j], pair 2g) and 64g + 32 + j (high nibble, pair 2g+1).
template <>
struct Dequant<QG_FMT_Q4K_RAW> {
  template <class Emit>
  __device__ __forceinline__ static void run(const uint8_t* blk, uint32_t h, uint32_t r, uint8_t* A2,
                                             const uint8_t*, Emit&& emit) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
#pragma unroll
    for (uint32_t gg = 0; gg < 2u; ++gg) {
      const uint32_t g = 2u * h + gg;
      uint32_t sc0, m0, sc1, m1;
      scale_min_k4(2u * g, hd.y, hd.z, hd.w, sc0, m0);
      scale_min_k4(2u * g + 1u, hd.y, hd.z, hd.w, sc1, m1);
      const float f0 = static_cast<float>(sc0), f1 = static_cast<float>(sc1);
      const __half2 s0 = __float2half2_rn(f0), c0 = __float2half2_rn(-1024.0f * f0);
      const __half2 s1 = __float2half2_rn(f1 * 0.0625f), c1 = __float2half2_rn(-64.0f * f1);
      const uint4* qs = reinterpret_cast<const uint4*>(blk + 16u + 32u * g);
      uint32_t lo[16], hi[16];
#pragma unroll
      for (uint32_t v = 0; v < 2u; ++v) {
        const uint4 q = qs[v];
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (uint32_t i = 0; i < 4u; ++i) {
          const uint32_t a0 = __byte_perm(w[i], 0, 0x4140), a1 = __byte_perm(w[i], 0, 0x4342);
          lo[8u * v + 2u * i] = hfma_bits(nib_lo(a0), s0, c0);
          lo[8u * v + 2u * i + 1u] = hfma_bits(nib_lo(a1), s0, c0);
          hi[8u * v + 2u * i] = hfma_bits(nib_hi(a0), s1, c1);
          hi[8u * v + 2u * i + 1u] = hfma_bits(nib_hi(a1), s1, c1);
        }
      }
      emit(2u * gg, lo);
      emit(2u * gg + 1u, hi);
    }
    if (h == 1u) store_mins(hd.y, hd.z, hd.w, r, A2);
  }
};

// Q5_K: block = d, dmin, scales[12], qh[32], qs[128]; q = nibble + 16 * bit, the bit of
// column 64g + j in qh[j] bit 2g (low part) or 2g+1 (high part).
template <>
struct Dequant<QG_FMT_Q5K> {
  template <class Emit>
  __device__ __forceinline__ static void run(const uint8_t* blk, uint32_t h, uint32_t r, uint8_t* A2,
                                             const uint8_t*, Emit&& emit) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const uint4* qhp = reinterpret_cast<const uint4*>(blk + 16u);
    const uint4 qh0 = qhp[0], qh1 = qhp[1];
    const uint32_t qhw[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
#pragma unroll
    for (uint32_t gg = 0; gg < 2u; ++gg) {
      const uint32_t g = 2u * h + gg;
      uint32_t sc0, m0, sc1, m1;
      scale_min_k4(2u * g, hd.y, hd.z, hd.w, sc0, m0);
      scale_min_k4(2u * g + 1u, hd.y, hd.z, hd.w, sc1, m1);
      const float f0 = static_cast<float>(sc0), f1 = static_cast<float>(sc1);
      const __half2 s0 = __float2half2_rn(f0), c0 = __float2half2_rn(-1024.0f * f0);
      const __half2 s1 = __float2half2_rn(f1 * 0.0625f), c1 = __float2half2_rn(-64.0f * f1);
      const uint4* qs = reinterpret_cast<const uint4*>(blk + 48u + 32u * g);
      const uint32_t sl = 2u * g, sh = 2u * g + 1u;
      uint32_t lo[16], hi[16];
#pragma unroll
      for (uint32_t v = 0; v < 2u; ++v) {
        const uint4 q = qs[v];
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (uint32_t i = 0; i < 4u; ++i) {
          const uint32_t qw = qhw[4u * v + i];  // qh bytes of the same 4 columns
#pragma unroll
          for (uint32_t s = 0; s < 2u; ++s) {
            const uint32_t sel = s == 0u ? 0x4140u : 0x4342u;
            const uint32_t pr = __byte_perm(w[i], 0, sel);
            const uint32_t hb = __byte_perm(qw, 0, sel);
            const uint32_t lo_h = nib_lo(pr) | (((hb >> sl) & 0x00010001u) << 4);
            const uint32_t hi_h = nib_hi(pr) | (((hb >> sh) & 0x00010001u) << 8);
            lo[8u * v + 2u * i + s] = hfma_bits(lo_h, s0, c0);
            hi[8u * v + 2u * i + s] = hfma_bits(hi_h, s1, c1);
          }
        }
      }
      emit(2u * gg, lo);
      emit(2u * gg + 1u, hi);
    }
    if (h == 1u) store_mins(hd.y, hd.z, hd.w, r, A2);
  }
};

// Little-endian 16-bit load from a 2-B aligned address.
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}
// n consecutive bytes (n multiple of 4) from a 2-B aligned address into words.
template <uint32_t N>
__device__ __forceinline__ void load_bytes(const uint8_t* p, uint32_t (&w)[N / 4]) {
#pragma unroll
  for (uint32_t i = 0; i < N / 4u; ++i) w[i] = lds_u16(p + 4u * i) | (lds_u16(p + 4u * i + 2u) << 16);
}

// IQ2_S: block = d, qs[64] (grid index low bits [0,32), signs [32,64)), qh[8], scales[8];
// group (ib32, g) = 8 columns: idx = qs[4 ib32 + g] | bits of qh[ib32], scale nibble
// low (g < 2) or high (g >= 2) of scales[ib32].  Shared tables: T2[idx] = the 8 grid
// magnitudes 2k+1 as fp16, SG[s] = 8 fp16 sign masks (0x8000 where bit j of s is set).
template <>
struct Dequant<QG_FMT_IQ2S> {
  template <class Emit>
  __device__ __forceinline__ static void run(const uint8_t* blk, uint32_t h, uint32_t, uint8_t*,
                                             const uint8_t* tables, Emit&& emit) {
    const uint4* t2 = reinterpret_cast<const uint4*>(tables);
    const uint4* sg = reinterpret_cast<const uint4*>(tables + 16384);
    uint32_t qs[4], sgn[4], qh[1], sc[1];
    load_bytes<16>(blk + 2u + 16u * h, qs);
    load_bytes<16>(blk + 34u + 16u * h, sgn);
    load_bytes<4>(blk + 66u + 4u * h, qh);
    load_bytes<4>(blk + 74u + 4u * h, sc);
#pragma unroll
    for (uint32_t i = 0; i < 4u; ++i) {  // ib32 = 4h + i
      const uint32_t hbits = byte_of(qh[0], i), sbyte = byte_of(sc[0], i);
      uint32_t o[16];
#pragma unroll
      for (uint32_t g = 0; g < 4u; ++g) {
        const uint32_t idx = byte_of(qs[i], g) | ((hbits << (8u - 2u * g)) & 0x300u);
        const uint32_t nib = g < 2u ? (sbyte & 15u) : (sbyte >> 4);
        const __half2 s = __float2half2_rn(static_cast<float>(2u * nib + 1u));
        const uint4 gv = t2[idx];
        const uint4 sm = sg[byte_of(sgn[i], g)];
        o[4u * g] = h2_bits(__hmul2(bits_h2(gv.x ^ sm.x), s));
        o[4u * g + 1u] = h2_bits(__hmul2(bits_h2(gv.y ^ sm.y), s));
        o[4u * g + 2u] = h2_bits(__hmul2(bits_h2(gv.z ^ sm.z), s));
        o[4u * g + 3u] = h2_bits(__hmul2(bits_h2(gv.w ^ sm.w), s));
      }
      emit(i, o);
    }
  }
};

// IQ3_S: block = d, qs[64], qh[8], signs[32], scales[4]; group (ib32, g) = 8 columns
// from two grid entries idx_p = qs[8 ib32 + 2g + p] | bit (2g + p) of qh[ib32] << 8,
// signs[4 ib32 + g], scale nibble of scales[ib32 / 2] (low for even ib32).  Shared
// tables: T3[idx] = the 4 grid magnitudes as fp16, SG as for IQ2_S.
template <>
struct Dequant<QG_FMT_IQ3S> {
  template <class Emit>
  __device__ __forceinline__ static void run(const uint8_t* blk, uint32_t h, uint32_t, uint8_t*,
                                             const uint8_t* tables, Emit&& emit) {
    const uint2* t3 = reinterpret_cast<const uint2*>(tables);
    const uint4* sg = reinterpret_cast<const uint4*>(tables + 4096);
    uint32_t qs[8], sgn[4], qh[1];
    load_bytes<32>(blk + 2u + 32u * h, qs);
    load_bytes<16>(blk + 74u + 16u * h, sgn);
    load_bytes<4>(blk + 66u + 4u * h, qh);
    const uint32_t scw = lds_u16(blk + 106u + 2u * h);  // scales of ib32 = 4h..4h+3
#pragma unroll
    for (uint32_t i = 0; i < 4u; ++i) {
      const uint32_t hbits = byte_of(qh[0], i);
      const uint32_t sb = byte_of(scw, i >> 1);
      const uint32_t nib = (i & 1u) == 0u ? (sb & 15u) : (sb >> 4);
      const __half2 s = __float2half2_rn(static_cast<float>(1u + 2u * nib));
      uint32_t o[16];
#pragma unroll
      for (uint32_t g = 0; g < 4u; ++g) {
        const uint32_t q2 = (qs[2u * i + (g >> 1)] >> (16u * (g & 1u))) & 0xffffu;
        const uint32_t i0 = (q2 & 0xffu) | (((hbits >> (2u * g)) & 1u) << 8);
        const uint32_t i1 = (q2 >> 8) | (((hbits >> (2u * g + 1u)) & 1u) << 8);
        const uint2 g0 = t3[i0], g1 = t3[i1];
        const uint4 sm = sg[byte_of(sgn[i], g)];
        o[4u * g] = h2_bits(__hmul2(bits_h2(g0.x ^ sm.x), s));
        o[4u * g + 1u] = h2_bits(__hmul2(bits_h2(g0.y ^ sm.y), s));
        o[4u * g + 2u] = h2_bits(__hmul2(bits_h2(g1.x ^ sm.z), s));
        o[4u * g + 3u] = h2_bits(__hmul2(bits_h2(g1.y ^ sm.w), s));
      }
      emit(i, o);
    }
  }
};

__device__ __forceinline__ uint32_t half_bits(float f) {
  return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(f)));
}

template <int FMT>
__device__ __forceinline__ void build_tables(uint8_t* t, uint32_t tid, uint32_t n) {
  if constexpr (FMT == QG_FMT_IQ2S) {
    uint4* t2 = reinterpret_cast<uint4*>(t);
    for (uint32_t i = tid; i < 1024u; i += n) {
      const uint32_t kg = g_iq2s_kgrid[i];
      uint32_t w[4];
#pragma unroll
      for (uint32_t j = 0; j < 4u; ++j) {
        const float a = static_cast<float>(2u * ((kg >> (4u * j)) & 3u) + 1u);
        const float b = static_cast<float>(2u * ((kg >> (4u * j + 2u)) & 3u) + 1u);
        w[j] = half_bits(a) | (half_bits(b) << 16);
      }
      t2[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else if constexpr (FMT == QG_FMT_IQ3S) {
    uint2* t3 = reinterpret_cast<uint2*>(t);
    for (uint32_t i = tid; i < 512u; i += n) {
      const uint32_t gw = g_iq3s_grid[i];
      t3[i] = make_uint2(half_bits(static_cast<float>(gw & 0xffu)) |
                             (half_bits(static_cast<float>((gw >> 8) & 0xffu)) << 16),
                         half_bits(static_cast<float>((gw >> 16) & 0xffu)) |
                             (half_bits(static_cast<float>(gw >> 24)) << 16));
    }
  }
  if constexpr (TcFmt<FMT>::window) {
    uint4* sg = reinterpret_cast<uint4*>(t + (FMT == QG_FMT_IQ2S ? 16384u : 4096u));
    for (uint32_t s = tid; s < 256u; s += n) {
      uint32_t w[4];
#pragma unroll
      for (uint32_t j = 0; j < 4u; ++j) {
        w[j] = (((s >> (2u * j)) & 1u) ? 0x8000u : 0u) | (((s >> (2u * j + 1u)) & 1u) ? 0x80000000u : 0u);
      }
      sg[s] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// ---------------------------------------------------------------------------

struct alignas(64) TcArgs {
  CUtensorMap tmap;      // payload as [rows][kb * bpb] bytes, box {row slot, 128}; valid if use_tmap
  const uint8_t* payload;
  const uint8_t* xrec;   // per block: fp16 x tile + sub-block sums (prepared)
  const float* xscale;   // per batch row: 2^e
  float* y;              // [batch, rows]
  float* partial;        // [grid][2][NB][128]
  uint32_t* counters;    // per row: contributions received (zeroed by the scale kernel)
  uint64_t units;        // tiles * kb
  uint64_t payload_bytes;
  uint32_t rows, kb, batch, grid, use_tmap;
};

__device__ __forceinline__ uint64_t range_start(uint64_t units, uint32_t grid, uint32_t c) {
  return units * c / grid;
}
// The CTA whose range holds unit u (ranges are never empty: grid <= units).
__device__ __forceinline__ uint32_t cta_of(uint64_t units, uint32_t grid, uint64_t u) {
  uint32_t c = static_cast<uint32_t>((u * grid) / units);
  if (c >= grid) c = grid - 1u;
  while (c + 1u < grid && range_start(units, grid, c + 1u) <= u) ++c;
  while (c > 0u && range_start(units, grid, c) > u) --c;
  return c;
}

template <int FMT, uint32_t NB>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ TcArgs args) {
  using F = TcFmt<FMT>;
  using L = TcLayout<FMT, NB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023));
  uint8_t* sA2 = sm + L::a2_off;
  uint8_t* sX = sm + L::x_off;
  uint8_t* sT = sm + L::t_off;
  uint8_t* sRaw = sm + L::raw_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::bar_off);
  constexpr uint32_t S = L::raw_stages;
  constexpr uint32_t kASlots = L::a_slots;
  constexpr uint32_t kTmemA = tmem_a<NB>();
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + S;
  static_assert(kXStages == kAccSlots, "x stages and accumulator slots share unit_done");
  uint64_t* a_full = raw_empty + S;        // per A slot: both dequantize halves written
  uint64_t* a_empty = a_full + kASlots;    // per A slot: its MMAs completed
  uint64_t* x_full = a_empty + kASlots;
  uint64_t* unit_done = x_full + kXStages; // per unit ring index: all MMAs of the unit completed
  uint64_t* acc_empty = unit_done + kXStages;
  uint64_t* done = acc_empty + kAccSlots;
  uint64_t* scale_full = done + 1;          // per accumulator slot: the unit's block scales written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(scale_full + kAccSlots);
  volatile uint32_t* abort = tmem_slot + 1;
  float* scales = reinterpret_cast<float*>(sm + L::bar_off + L::scl_rel);

  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  const uint64_t u0 = range_start(args.units, args.grid, blockIdx.x);
  const uint64_t u1 = range_start(args.units, args.grid, blockIdx.x + 1u);
  const uint32_t n_units = static_cast<uint32_t>(u1 - u0);
  const uint32_t kb = args.kb;

  if (tid == 0) {
    for (uint32_t i = 0; i < S; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 8);  // one arrival per dequant warp
    }
    for (uint32_t i = 0; i < kASlots; ++i) {
      mbar_init(&a_full[i], 256);   // every dequantize thread
      mbar_init(&a_empty[i], 1);    // MMA commit
    }
    for (uint32_t i = 0; i < kXStages; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&unit_done[i], 1);  // MMA commit: frees the x stage, fills the accumulator
      mbar_init(&acc_empty[i], 4);  // one arrival per epilogue warp
    }
    mbar_init(done, 1);
    for (uint32_t i = 0; i < kAccSlots; ++i) mbar_init(&scale_full[i], 4);  // the h = 0 dequantize warps
    *abort = 0u;
    fence_mbar_init();
  }
  if (warp == 1u) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if constexpr (F::window) {
    if (warp >= kDequantWarp0) build_tables<FMT>(sT, tid - 64u, kThreads - 64u);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0u) {
    // ---------------- weight producer ----------------
    const uint64_t policy = l2_evict_first_policy();
    const uint64_t aligned_end = args.payload_bytes & ~uint64_t(15);
    uint32_t issued = 0;
    for (uint32_t n = 0; n < n_units; ++n) {
      const uint64_t u = u0 + n;
      const uint32_t tile = static_cast<uint32_t>(u / kb), k = static_cast<uint32_t>(u % kb);
      const uint32_t s = n % S;
      if (n >= S && !tc_wait_warp(&raw_empty[s], ((n / S) & 1u) ^ 1u, abort, lane)) break;
      uint8_t* stage = sRaw + s * L::raw_stage;
      if (args.use_tmap) {
        if (lane == 0u) {
          mbar_arrive_expect_tx(&raw_full[s], L::raw_stage);
          const uint32_t x0 = (k * F::bpb) & ~15u;
          tma_load_2d(stage, &args.tmap, static_cast<int32_t>(x0), static_cast<int32_t>(tile * kTileM),
                      &raw_full[s], policy);
        }
        __syncwarp();
      } else {
        uint64_t src[4];
        uint32_t len[4];
        uint32_t bytes = 0;
#pragma unroll
        for (uint32_t i = 0; i < 4u; ++i) {
          const uint32_t r = lane + 32u * i, row = tile * kTileM + r;
          len[i] = 0;
          src[i] = 0;
          if (row < args.rows) {
            const uint64_t a = (static_cast<uint64_t>(row) * kb + k) * F::bpb;
            if constexpr (F::window) {
              const uint64_t s0 = a & ~uint64_t(15);
              uint64_t e = (a + F::bpb + 15u) & ~uint64_t(15);
              if (e > aligned_end) {
                // the payload's unaligned last bytes: copied with plain loads here
                e = aligned_end;
                const uint64_t from = a > aligned_end ? a : aligned_end;
                for (uint64_t b = from; b < a + F::bpb; ++b) {
                  stage[r * F::rowb + (b - s0)] = args.payload[b];
                }
              }
              src[i] = s0;
              len[i] = e > s0 ? static_cast<uint32_t>(e - s0) : 0u;
            } else {
              src[i] = a;
              len[i] = F::bpb;
            }
            bytes += len[i];
          }
        }
        const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
        __syncwarp();
        if (lane == 0u) mbar_arrive_expect_tx(&raw_full[s], total);
        __syncwarp();
#pragma unroll
        for (uint32_t i = 0; i < 4u; ++i) {
          if (len[i] != 0u) {
            tma_load_1d(stage + (lane + 32u * i) * F::rowb, args.payload + src[i], len[i], &raw_full[s],
                        policy);
          }
        }
      }
      ++issued;
    }
    // drain: every copy issued must have landed before the CTA exits
    if (lane == 0u) {
      const uint32_t rs = issued < S ? issued : S;
      for (uint32_t i = 0; i < rs; ++i) {
        const uint32_t n = issued - 1u - i;
        mbar_wait_bounded(&raw_full[n % S], (n / S) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == kXWarp) {
    // ---------------- x producer ----------------
    pdl_wait();  // the prepared x is the previous kernel's output
    uint32_t issued = 0;
    for (uint32_t n = 0; n < n_units; ++n) {
      const uint32_t k = static_cast<uint32_t>((u0 + n) % kb);
      const uint32_t xs = n % kXStages;
      if (n >= kXStages && !tc_wait_warp(&unit_done[xs], ((n / kXStages) & 1u) ^ 1u, abort, lane)) break;
      if (lane == 0u) {
        mbar_arrive_expect_tx(&x_full[xs], L::xrec);
        tma_load_1d(sX + xs * L::xrec, args.xrec + static_cast<uint64_t>(k) * L::xrec, L::xrec, &x_full[xs]);
      }
      __syncwarp();
      ++issued;
    }
    if (lane == 0u) {
      const uint32_t xsn = issued < kXStages ? issued : kXStages;
      for (uint32_t i = 0; i < xsn; ++i) {
        const uint32_t n = issued - 1u - i;
        mbar_wait_bounded(&x_full[n % kXStages], (n / kXStages) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1u) {
    // ---------------- MMA issuer ----------------
    if (lane == 0u) {
      constexpr uint32_t idesc = umma_idesc<NB>();
      const uint32_t a2_base = smem_addr(sA2), x_base = smem_addr(sX);
      for (uint32_t n = 0; n < n_units; ++n) {
        const uint32_t t = n % kAccSlots, as = n % kASlots;
        // accumulator slot free, x landed, A slot written: three independent polls
        if (!tc_spin3(n >= kAccSlots ? &acc_empty[t] : nullptr, ((n / kAccSlots) & 1u) ^ 1u, &x_full[t],
                      (n / kXStages) & 1u, &a_full[as], (n / kASlots) & 1u, abort)) {
          break;
        }
        tc_fence_after();
        const uint32_t d_q = tmem + t * 2u * NB, d_m = d_q + NB;
        const uint32_t xb = x_base + t * L::xrec;
        const uint32_t a_t = tmem + kTmemA + as * 128u;
#pragma unroll
        for (uint32_t j = 0; j < 16u; ++j) {
          umma_ts(d_q, a_t + 8u * j, umma_desc(xb + j * (NB * 32u)), idesc, j != 0u ? 1u : 0u);
        }
        if constexpr (F::has_min) {
          umma_ss(d_m, umma_desc(a2_base + as * kA2Bytes), umma_desc(xb + NB * 512u), idesc, 0u);
        }
        umma_commit(&a_empty[as]);
        umma_commit(&unit_done[t]);
      }
      // every MMA issued must have completed before tensor memory is freed
      umma_commit(done);
      mbar_wait_bounded(done, 0);
    }
    __syncwarp();
  } else if (warp < kEpilogueWarp0) {
    // ---------------- dequantize ----------------
    const uint32_t h = (warp - kDequantWarp0) >> 2, quarter = warp & 3u;
    const uint32_t r = quarter * 32u + lane;
    const uint32_t lane_addr = (quarter * 32u) << 16;
    for (uint32_t n = 0; n < n_units; ++n) {
      const uint64_t u = u0 + n;
      const uint32_t tile = static_cast<uint32_t>(u / kb), k = static_cast<uint32_t>(u % kb);
      const uint32_t row = tile * kTileM + r;
      const uint32_t s = n % S, as = n % kASlots;
      if (!tc_wait_warp(&raw_full[s], (n / S) & 1u, abort, lane)) break;
      if (n >= kASlots && !tc_wait_warp(&a_empty[as], ((n / kASlots) & 1u) ^ 1u, abort, lane)) break;
      tc_fence_after();
      const uint32_t a_t = tmem + lane_addr + kTmemA + as * 128u + h * 64u;
      uint8_t* A2 = sA2 + as * kA2Bytes;
      auto emit = [&](uint32_t g, const uint32_t (&w)[16]) { tmem_st16(a_t + 16u * g, w); };
      // every lane runs the (warp-collective) tensor-memory stores: rows past the matrix
      // dequantize whatever their slot holds, and their results are never written
      uint32_t off = 0;
      if constexpr (F::window) off = static_cast<uint32_t>(((static_cast<uint64_t>(row) * kb + k) * F::bpb) & 15u);
      const uint8_t* blk = sRaw + s * L::raw_stage + r * F::rowb + off;
      if (h == 0u) {
        // The unit's block scales for the epilogue, from the staged block (the weight
        // stream is L2 evict-first, so re-reading them from global memory would go to
        // DRAM once per row and unit).  Slot t is free once the epilogue released unit
        // n - kAccSlots.
        const uint32_t t = n % kAccSlots;
        if (n >= kAccSlots && !tc_wait_warp(&acc_empty[t], ((n / kAccSlots) & 1u) ^ 1u, abort, lane)) break;
        const float d = h2f(lds_u16(blk));
        scales[(t * 2u) * kTileM + r] = FMT == QG_FMT_IQ2S ? d * 0.125f : d;
        scales[(t * 2u + 1u) * kTileM + r] = F::has_min ? h2f(lds_u16(blk + 2)) : 0.f;
        __syncwarp();
        if (lane == 0u) mbar_arrive(&scale_full[t]);
      }
      Dequant<FMT>::run(blk, h, r, A2, sT, emit);
      tmem_wait_st();
      if (F::has_min && h == 1u) fence_proxy_async_smem();  // min tile -> tensor core
      tc_fence_before();
      mbar_arrive(&a_full[as]);
      __syncwarp();
      if (lane == 0u) mbar_arrive(&raw_empty[s]);
    }
  } else {
    // ---------------- epilogue ----------------
    pdl_wait();
    const uint32_t quarter = warp & 3u;  // tensor-memory lanes this warp may read
    const uint32_t r = quarter * 32u + lane;
    const uint32_t first_tile = static_cast<uint32_t>(u0 / kb);
    float y[NB];
#pragma unroll
    for (uint32_t b = 0; b < NB; ++b) y[b] = 0.f;
    for (uint32_t n = 0; n < n_units; ++n) {
      const uint64_t u = u0 + n;
      const uint32_t tile = static_cast<uint32_t>(u / kb), k = static_cast<uint32_t>(u % kb);
      const uint32_t row = tile * kTileM + r;
      const uint32_t t = n % kAccSlots;
      if (!tc_wait_warp(&unit_done[t], (n / kAccSlots) & 1u, abort, lane)) break;
      if (!tc_wait_warp(&scale_full[t], (n / kAccSlots) & 1u, abort, lane)) break;
      tc_fence_after();
      // block scales of the unit's rows (written by the dequantize warps)
      const float dq = scales[(t * 2u) * kTileM + r];
      const float dm = F::has_min ? scales[(t * 2u + 1u) * kTileM + r] : 0.f;
      const uint32_t taddr = tmem + ((quarter * 32u) << 16) + t * 2u * NB;
#pragma unroll
      for (uint32_t c = 0; c < NB; c += 16u) {
        float aq[16], am[16];
        tmem_ld16(taddr + c, aq);
        if constexpr (F::has_min) tmem_ld16(taddr + NB + c, am);
        tmem_wait_ld();
        if (c + 16u == NB) {
          // this warp's accumulator columns are all in registers: release the slot
          tc_fence_before();
          __syncwarp();
          if (lane == 0u) mbar_arrive(&acc_empty[t]);
        }
#pragma unroll
        for (uint32_t b = 0; b < 16u; ++b) {
          y[c + b] += F::has_min ? fmaf(dq, aq[b], -dm * am[b]) : dq * aq[b];
        }
      }
      if (k == kb - 1u || n == n_units - 1u) {
        // the CTA's last unit of this tile: publish the tile's rows
        const uint64_t tu0 = static_cast<uint64_t>(tile) * kb;
        const bool full = u0 <= tu0 && u1 >= tu0 + kb;
        if (row < args.rows) {
          if (full) {
#pragma unroll
            for (uint32_t b = 0; b < NB; ++b) {
              if (b < args.batch) args.y[static_cast<uint64_t>(b) * args.rows + row] = y[b] * args.xscale[b];
            }
          } else {
            const uint32_t j = tile == first_tile ? 0u : 1u;
            float* P = args.partial + (static_cast<uint64_t>(blockIdx.x) * 2u + j) * NB * kTileM;
#pragma unroll
            for (uint32_t b = 0; b < NB; ++b) P[b * kTileM + r] = y[b];
            __threadfence();
            const uint32_t c_first = cta_of(args.units, args.grid, tu0);
            const uint32_t c_last = cta_of(args.units, args.grid, tu0 + kb - 1u);
            const uint32_t old = atomicAdd(&args.counters[row], 1u);
            if (old == c_last - c_first) {
              // last contribution to this row: sum all of them in CTA order
              __threadfence();
              float acc[NB];
#pragma unroll
              for (uint32_t b = 0; b < NB; ++b) acc[b] = 0.f;
              for (uint32_t c = c_first; c <= c_last; ++c) {
                const uint32_t jc =
                    tile == static_cast<uint32_t>(range_start(args.units, args.grid, c) / kb) ? 0u : 1u;
                const float* Pc = args.partial + (static_cast<uint64_t>(c) * 2u + jc) * NB * kTileM;
#pragma unroll
                for (uint32_t b = 0; b < NB; ++b) {
                  acc[b] += c == blockIdx.x ? y[b] : __ldcg(Pc + b * kTileM + r);
                }
              }
#pragma unroll
              for (uint32_t b = 0; b < NB; ++b) {
                if (b < args.batch) args.y[static_cast<uint64_t>(b) * args.rows + row] = acc[b] * args.xscale[b];
              }
            }
          }
        }
#pragma unroll
        for (uint32_t b = 0; b < NB; ++b) y[b] = 0.f;
      }
    }
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1u) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

// Per batch row b: 2^e with max|x_b| <= 2^e (xscale[b] = 2^(e-10), so that
// xh = x / xscale has max|xh| <= 1024); padding rows get 1.  Also zeroes the per-row
// counters of the stream-K fixup.  One CTA of 256 threads per batch row.
template <uint32_t NB>
__global__ void __launch_bounds__(256) gemm_tc_scale_kernel(const float* __restrict__ x, uint32_t batch,
                                                            uint32_t cols, float* xscale,
                                                            uint32_t* counters, uint32_t n_counters) {
  __shared__ float wmax[8];
  pdl_wait();
  pdl_trigger();
  const uint32_t b = blockIdx.x, tid = threadIdx.x;
  for (uint32_t i = b * 256u + tid; i < n_counters; i += gridDim.x * 256u) counters[i] = 0u;
  if (b == 0u) {
    for (uint32_t i = batch + tid; i < NB; i += 256u) xscale[i] = 1.0f;
  }
  float m = 0.f;
  const float* xr = x + static_cast<uint64_t>(b) * cols;
  for (uint32_t c = tid; c < cols; c += 256u) m = fmaxf(m, fabsf(xr[c]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31u) == 0u) wmax[tid >> 5] = m;
  __syncthreads();
  if (tid == 0u) {
    m = wmax[0];
    for (uint32_t w = 1; w < 8u; ++w) m = fmaxf(m, wmax[w]);
    int e = 0;
    if (m > 0.f && m <= 3.4028234663852886e38f) {
      frexpf(m, &e);  // m < 2^e
      if (e < -100) e = -100;
    }
    xscale[b] = ldexpf(1.0f, e - 10);
  }
}

// x [batch, cols] fp32 -> per 256-column block k: the fp16 tile xh = x / xscale[b] in
// the UMMA layout and the 32-column sub-block sums of xh as fp16 hi + lo.  CTA
// (k, group of 8 batch rows); warp w = batch row, lane = 8 consecutive columns.
template <uint32_t NB>
__global__ void __launch_bounds__(256) gemm_tc_prep_kernel(const float* __restrict__ x, uint32_t batch,
                                                           uint32_t cols, const float* xscale,
                                                           uint8_t* xrec) {
  pdl_wait();
  pdl_trigger();
  const uint32_t k = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t b = blockIdx.y * 8u + warp, c0 = lane * 8u;
  float v[8];
  if (b < batch) {
    const float inv = 1.0f / xscale[b];  // a power of two: exact
    const float* xr = x + static_cast<uint64_t>(b) * cols + k * kBlockCols + c0;
#pragma unroll
    for (uint32_t i = 0; i < 8u; ++i) v[i] = xr[i] * inv;
  } else {
#pragma unroll
    for (uint32_t i = 0; i < 8u; ++i) v[i] = 0.f;
  }
  uint32_t h[4];
  float s = 0.f;
#pragma unroll
  for (uint32_t i = 0; i < 4u; ++i) {
    const __half2 p = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    h[i] = h2_bits(p);
    s += __low2float(p);
    s += __high2float(p);
  }
  uint8_t* rec = xrec + static_cast<uint64_t>(k) * (NB * 544u);
  *reinterpret_cast<uint4*>(rec + x_elem<NB>(b, c0)) = make_uint4(h[0], h[1], h[2], h[3]);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  if ((lane & 3u) == 0u) {
    const __half hi = __float2half_rn(s);
    const __half lo = __float2half_rn(s - __half2float(hi));
    const uint32_t o = NB * 512u + (b >> 3) * 256u + (b & 7u) * 16u + (lane >> 2) * 2u;
    *reinterpret_cast<__half*>(rec + o) = hi;
    *reinterpret_cast<__half*>(rec + o + 128u) = lo;
  }
}

size_t align256(size_t v) { return (v + 255u) & ~size_t(255); }

struct TcWorkspace {
  size_t xrec, xscale, partial, counters, total;
};

TcWorkspace tc_workspace(uint32_t nb, uint32_t rows, uint32_t cols, uint32_t grid) {
  const uint32_t kb = cols / kBlockCols;
  const uint32_t tiles = (rows + kTileM - 1u) / kTileM;
  TcWorkspace w{};
  size_t off = 0;
  w.xrec = off;
  off = align256(off + static_cast<size_t>(kb) * nb * 544u);
  w.xscale = off;
  off = align256(off + static_cast<size_t>(nb) * 4u);
  w.partial = off;
  off = align256(off + static_cast<size_t>(grid) * 2u * nb * kTileM * 4u);
  w.counters = off;
  off = align256(off + static_cast<size_t>(tiles) * kTileM * 4u);
  w.total = off;
  return w;
}

cudaError_t sm_count(int* n) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  return cudaDeviceGetAttribute(n, cudaDevAttrMultiProcessorCount, dev);
}

bool tc_format(int fmt) {
  return fmt == QG_FMT_Q4K_RAW || fmt == QG_FMT_Q5K || fmt == QG_FMT_IQ2S || fmt == QG_FMT_IQ3S;
}

// Partial-sum slots in the workspace: one pair per CTA of a grid of at most kMaxTcGrid
// CTAs, so the workspace size does not depend on the device the size was queried on
// (the launch grid is min(units, SMs, kMaxTcGrid)).
constexpr uint32_t kMaxTcGrid = 256u;

uint32_t grid_for(uint32_t sms, uint64_t units) {
  const uint32_t cap = sms < kMaxTcGrid ? sms : kMaxTcGrid;
  return units < cap ? static_cast<uint32_t>(units) : cap;
}

std::mutex g_attr_mutex;
std::set<std::pair<const void*, int>> g_attr_done;

template <typename K>
cudaError_t ensure_smem(K kernel, uint32_t bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  if (g_attr_done.count(key)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) g_attr_done.insert(key);
  return e;
}

template <int FMT, uint32_t NB>
cudaError_t launch_tc(const TcArgs& a, cudaStream_t stream) {
  using L = TcLayout<FMT, NB>;
  auto kernel = gemm_tc_kernel<FMT, NB>;
  cudaError_t e = ensure_smem(kernel, L::smem);
  if (e != cudaSuccess) return e;
  return launch_k(kernel, a.grid, kThreads, L::smem, stream, a);
}

template <uint32_t NB>
cudaError_t launch_tc_fmt(int fmt, const TcArgs& a, cudaStream_t stream) {
  switch (fmt) {
    case QG_FMT_Q4K_RAW: return launch_tc<QG_FMT_Q4K_RAW, NB>(a, stream);
    case QG_FMT_Q5K: return launch_tc<QG_FMT_Q5K, NB>(a, stream);
    case QG_FMT_IQ2S: return launch_tc<QG_FMT_IQ2S, NB>(a, stream);
    case QG_FMT_IQ3S: return launch_tc<QG_FMT_IQ3S, NB>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

// cuTensorMapEncodeTiled from the driver (looked up once; no link-time dependency on
// libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      p = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// The payload as a 2-D byte tensor [rows][kb * bpb] with a {row_slot, 128} box, when the
// row stride is a 16-B multiple and the matrix covers one box; false otherwise.
bool encode_payload_map(CUtensorMap* map, const uint8_t* payload, uint32_t rows, uint32_t kb,
                        uint32_t bpb, uint32_t row_slot) {
  const uint64_t row_bytes = static_cast<uint64_t>(kb) * bpb;
  if (row_bytes % 16u != 0u || rows < kTileM || row_bytes < row_slot || row_bytes >= (1ull << 32)) {
    return false;
  }
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {row_slot, kTileM};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(payload), dims, strides, box,
                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

uint32_t gemm_tc_nb(uint32_t batch) { return batch <= 16u ? 16u : 32u; }

// Independent of the current device (no CUDA call): sized for the largest grid.
cudaError_t gemm_tc_workspace_bytes(uint32_t batch, uint32_t rows, uint32_t cols, size_t* bytes) {
  const uint64_t units = static_cast<uint64_t>((rows + kTileM - 1u) / kTileM) * (cols / kBlockCols);
  *bytes = tc_workspace(gemm_tc_nb(batch), rows, cols, grid_for(kMaxTcGrid, units)).total;
  return cudaSuccess;
}

// Y = X W^T on the tensor cores (arguments validated by the caller).
cudaError_t launch_gemm_tc(int fmt, const uint8_t* payload, const float* x, float* y, uint32_t batch,
                           uint32_t rows, uint32_t cols, void* workspace, cudaStream_t stream) {
  int sms = 0;
  cudaError_t e = sm_count(&sms);
  if (e != cudaSuccess) return e;
  const uint32_t nb = gemm_tc_nb(batch);
  const uint32_t kb = cols / kBlockCols;
  const uint32_t tiles = (rows + kTileM - 1u) / kTileM;
  const uint64_t units = static_cast<uint64_t>(tiles) * kb;
  const uint32_t grid = grid_for(static_cast<uint32_t>(sms), units);
  const TcWorkspace w = tc_workspace(nb, rows, cols, grid_for(kMaxTcGrid, units));
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  TcArgs a{};
  a.payload = payload;
  a.xrec = ws + w.xrec;
  a.xscale = reinterpret_cast<const float*>(ws + w.xscale);
  a.y = y;
  a.partial = reinterpret_cast<float*>(ws + w.partial);
  a.counters = reinterpret_cast<uint32_t*>(ws + w.counters);
  a.units = units;
  a.rows = rows;
  a.kb = kb;
  a.batch = batch;
  a.grid = grid;
  const uint32_t bpb = fmt == QG_FMT_Q4K_RAW ? 144u : fmt == QG_FMT_Q5K ? 176u : fmt == QG_FMT_IQ2S ? 82u : 110u;
  const uint32_t row_slot = fmt == QG_FMT_Q4K_RAW ? TcFmt<QG_FMT_Q4K_RAW>::rowb
                            : fmt == QG_FMT_Q5K  ? TcFmt<QG_FMT_Q5K>::rowb
                            : fmt == QG_FMT_IQ2S ? TcFmt<QG_FMT_IQ2S>::rowb
                                                 : TcFmt<QG_FMT_IQ3S>::rowb;
  a.payload_bytes = static_cast<uint64_t>(rows) * kb * bpb;
  a.use_tmap = encode_payload_map(&a.tmap, payload, rows, kb, bpb, row_slot) ? 1u : 0u;
  const uint32_t n_counters = tiles * kTileM;
  float* xscale = reinterpret_cast<float*>(ws + w.xscale);
  if (nb == 16u) {
    e = launch_k(gemm_tc_scale_kernel<16>, batch, 256, 0, stream, x, batch, cols, xscale, a.counters, n_counters);
    if (e == cudaSuccess) {
      e = launch_k(gemm_tc_prep_kernel<16>, dim3(kb, 2), 256, 0, stream, x, batch, cols,
                   static_cast<const float*>(xscale), ws + w.xrec);
    }
    return e != cudaSuccess ? e : launch_tc_fmt<16>(fmt, a, stream);
  }
  e = launch_k(gemm_tc_scale_kernel<32>, batch, 256, 0, stream, x, batch, cols, xscale, a.counters, n_counters);
  if (e == cudaSuccess) {
    e = launch_k(gemm_tc_prep_kernel<32>, dim3(kb, 4), 256, 0, stream, x, batch, cols,
                 static_cast<const float*>(xscale), ws + w.xrec);
  }
  return e != cudaSuccess ? e : launch_tc_fmt<32>(fmt, a, stream);
}

bool gemm_tc_supports(int fmt) { return tc_format(fmt); }

bool batched_uses_tc(int fmt, const uint8_t* payload, uint32_t batch) {
  return batch >= tc_min_batch() && tc_format(fmt) && (reinterpret_cast<uintptr_t>(payload) & 15u) == 0u;
}

size_t batched_gemm_ws_bytes(int fmt, uint32_t batch, uint32_t rows, uint32_t cols) {
  if (batch < tc_min_batch() || !tc_format(fmt)) return 0u;
  size_t bytes = 0;
  gemm_tc_workspace_bytes(batch, rows, cols, &bytes);
  return bytes;
}

cudaError_t launch_batched_gemm(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                                float* y, uint32_t batch, uint32_t rows, uint32_t cols,
                                void* workspace, cudaStream_t stream) {
  if (workspace != nullptr && batched_uses_tc(fmt, payload, batch)) {
    return launch_gemm_tc(fmt, payload, x, y, batch, rows, cols, workspace, stream);
  }
  return launch_gemv_vectors(fmt, payload, meta, x, y, batch, rows, cols, stream);
}

// First batch size qg_gemm_batched runs on the tensor cores: kTcMinBatch, or the
// QG_TC_MIN_BATCH environment variable (2..33; 33 keeps every batch on the CUDA cores),
// read once per process.
uint32_t tc_min_batch() {
  static const uint32_t v = [] {
    const char* e = std::getenv("QG_TC_MIN_BATCH");
    if (e == nullptr) return kTcMinBatch;
    const long n = std::strtol(e, nullptr, 10);
    return n >= 2 && n <= 33 ? static_cast<uint32_t>(n) : kTcMinBatch;
  }();
  return v;
}

}  // namespace qg

extern "C" {

cudaError_t qg_gemm_batched_workspace_bytes(int fmt, uint32_t batch, uint32_t rows, uint32_t cols,
                                            size_t* bytes) {
  if (bytes == nullptr || !qg::gemm_tc_supports(fmt) || batch == 0u || batch > 32u || rows == 0u ||
      cols == 0u || cols % 256u != 0u) {
    return cudaErrorInvalidValue;
  }
  return qg::gemm_tc_workspace_bytes(batch, rows, cols, bytes);
}

cudaError_t qg_gemm_batched(int fmt, const uint8_t* payload, const uint8_t* meta, const float* x,
                            float* y, uint32_t batch, uint32_t rows, uint32_t cols, void* workspace,
                            cudaStream_t stream) {
  (void)meta;
  if (!qg::gemm_tc_supports(fmt) || payload == nullptr || x == nullptr || y == nullptr ||
      workspace == nullptr || batch == 0u || batch > 32u || rows == 0u || cols == 0u ||
      cols % 256u != 0u || (reinterpret_cast<uintptr_t>(payload) & 15u) != 0u ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0u) {
    return cudaErrorInvalidValue;
  }
  // Below the tensor-core threshold the CUDA-core multi-vector GEMV reads each weight once
  // for up to 8 vectors (qg_gemv_batch.cu); the tensor-core tiles take larger batches.
  if (batch < qg::tc_min_batch()) {
    return qg::launch_gemv_vectors(fmt, payload, meta, x, y, batch, rows, cols, stream);
  }
  return qg::launch_gemm_tc(fmt, payload, x, y, batch, rows, cols, workspace, stream);
}

}  // extern "C"
