// common.cuh — device helpers shared by the sm_100a kernels: mbarriers, bulk
// (TMA) copies, bounded waits, and the bit-exact scalar steps of the
// reference's arithmetic.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mri_gpu.h"

namespace mri {

// A bounded wait gives up after this many SM clocks (~1 s at 1.9 GHz) and
// reports MRI_ERR_TIMEOUT through the context's device status word.
constexpr long long kWaitBudgetClocks = 2000000000LL;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
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
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false (and
// records MRI_ERR_TIMEOUT in *status) if the budget runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > kWaitBudgetClocks) {
      if (status) *reinterpret_cast<volatile int*>(status) = MRI_ERR_TIMEOUT;
      return false;
    }
  }
}

// Bulk prefetch of [src, src + bytes) into L2 (src 16-byte aligned, bytes a
// multiple of 16).  A hint: no completion, no effect on results.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 1-D bulk copy global -> shared, completing `bytes` of transaction count on
// `bar`.  dst and src 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Same, with an L2 evict-first policy for data streamed exactly once.
__device__ __forceinline__ void bulk_copy_g2s_stream(void* dst, const void* src, uint32_t bytes,
                                                     uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
      "%2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Loads of data that an earlier kernel in the stream wrote (activations, the
// KV cache, gathered slices).  Kernels here start early under programmatic
// dependent launch, so the SM's L1 can hold lines of these buffers from
// before the producer kernel rewrote them; the non-coherent read-only path
// (ld.global.nc) could return such stale lines.  These loads are cached in
// L2 only.
template <typename T>
__device__ __forceinline__ T ld_act(const T* p) { return __ldcg(p); }

// Named barrier among `threads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
  return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// ── bit-exact steps of the reference arithmetic ────────────────────────────

// symmetric.rs:46: scale = max_abs == 0 ? 1 : max_abs / 127 (IEEE division).
__device__ __forceinline__ float sym_scale(float max_abs) {
  return max_abs == 0.0f ? 1.0f : __fdiv_rn(max_abs, 127.0f);
}

// symmetric.rs:51-54: q = clamp(round(v * inv), -127, 127) as i8.  round is
// half-away-from-zero (roundf); `as i8` maps NaN to 0.
__device__ __forceinline__ int8_t sym_quant(float v, float inv) {
  const float r = roundf(__fmul_rn(v, inv));
  if (r != r) return 0;
  return static_cast<int8_t>(fminf(fmaxf(r, -127.0f), 127.0f));
}

// int8.rs:93: `acc as f32 * act_scale * scales[n]`, left to right.
__device__ __forceinline__ float rescale(int acc, float s_a, float s_w) {
  return __fmul_rn(__fmul_rn(__int2float_rn(acc), s_a), s_w);
}

// (f32)v for |v| < 2^22 without the conversion unit: v added to the bit
// pattern of 1.5 * 2^23 lands in the mantissa of a float in [2^23, 2^24),
// whose value is exactly 1.5 * 2^23 + v; subtracting 1.5 * 2^23 is exact too.
// Equal to __int2float_rn(v) in that range (a Q8_0 block dot is at most
// 32 * 127 * 127 in magnitude).
__device__ __forceinline__ float small_int_to_float(int v) {
  return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}

// f16_to_f32 (gguf/quantization.rs:416-461) is the exact IEEE conversion.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

// Max of |v| over a value set, NaN-skipping (fold(0.0, f32::max)).
__device__ __forceinline__ float absmax_acc(float m, float v) { return fmaxf(m, fabsf(v)); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace mri
