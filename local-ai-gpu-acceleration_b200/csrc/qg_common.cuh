// qg_common.cuh -- device helpers shared by the sm_100a decode kernels.
//
//  * 1-D TMA (cp.async.bulk, plain form) into shared memory with mbarrier
//    completion, and bounded mbarrier waits that record QG_ERR_WAIT_TIMEOUT in the
//    library's error word instead of spinning forever.
//  * Field decoders for the GGUF super-blocks: fp16 scale words and the 6-bit
//    K-quant (scale, min) pairs.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qgemv_b200.h"

namespace qg {

// Library-wide device error word (QG_ERR_* bits); read and cleared by qg_get_error.
extern __device__ unsigned int g_error_word;

constexpr uint32_t kMaxSpin = 1u << 22;  // bounded mbarrier polls before giving up

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0u;
}

// Bounded wait for phase `parity` of `bar`.  Returns false (and sets the error word)
// when the poll budget runs out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t it = 0; it < kMaxSpin; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  atomicOr(&g_error_word, QG_ERR_WAIT_TIMEOUT);
  return false;
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-B aligned),
// completing on `bar`.  Plain form: the source is this GPU's own memory.
// L2 evict-first: weights are streamed once per call.
__device__ __forceinline__ void tma_load_1d(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Same without an L2 cache hint.
__device__ __forceinline__ void tma_load_1d(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// Programmatic dependent launch.  pdl_wait: block until the grids this one depends on
// have completed and their writes are visible (a no-op without a programmatic edge);
// every kernel calls it before reading another kernel's output or writing global
// memory -- only immutable data (the weights) may be read before it.  pdl_trigger:
// allow the dependent grid to start launching (its CTAs then run their own
// pre-wait prologue while this grid finishes).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// System-scope relaxed 64-bit store / load (single-copy atomic when 8-B aligned): words
// exchanged with other GPUs over NVLink, each carrying its own epoch.
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// IEEE fp16 bit pattern -> fp32 (exact for every finite value; the reference's
// fp16_bits_to_float, decode_kernels.cu:1665-1676, gives the same value).
__device__ __forceinline__ float h2f(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, uint32_t i) { return (w >> (8u * i)) & 0xffu; }

// get_scale_min_k4 (decode_kernels.cu:1678-1692) for pair index j in 0..7 of the
// 12 packed bytes held little-endian in (s0, s1, s2) = bytes 0-3, 4-7, 8-11.
__device__ __forceinline__ void scale_min_k4(uint32_t j, uint32_t s0, uint32_t s1, uint32_t s2,
                                             uint32_t& sc, uint32_t& mn) {
  const uint32_t k = j & 3u;
  if (j < 4u) {
    sc = byte_of(s0, k) & 63u;
    mn = byte_of(s1, k) & 63u;
  } else {
    const uint32_t b8 = byte_of(s2, k);  // packed[j + 4]
    sc = (b8 & 0x0fu) | ((byte_of(s0, k) >> 6u) << 4u);
    mn = (b8 >> 4u) | ((byte_of(s1, k) >> 6u) << 4u);
  }
}

// 2^23 + b for a byte b placed in the low mantissa bits: a float whose value minus
// 2^23 is exactly b.  sel picks the byte of w (0..3).
__device__ __forceinline__ float byte_magic(uint32_t w, uint32_t sel) {
  return __uint_as_float(__byte_perm(w, 0x4b000000u, 0x7650u | sel));
}

constexpr float kMagic = 8388608.0f;  // 2^23

// Compile-time byte sizes of a format's payload and metadata streams per block.
template <int FMT>
struct FmtTraits {
  static constexpr uint32_t payload_bytes =
      FMT == QG_FMT_Q4K_RAW ? 144u : FMT == QG_FMT_Q5K ? 176u : FMT == QG_FMT_IQ2S ? 82u
      : FMT == QG_FMT_IQ3S ? 110u : 128u;
  static constexpr uint32_t meta_bytes =
      FMT == QG_FMT_Q4K_SPLIT_PREDECODED ? 64u : FMT == QG_FMT_Q4K_SPLIT_HALF ? 32u
      : FMT == QG_FMT_Q4K_SPLIT_COMPACT ? 20u : FMT == QG_FMT_Q4K_SPLIT_NATIVE ? 16u : 0u;
};

}  // namespace qg
