// quant.cu — K1: symmetric INT8 activation quantizer (quantize_symmetric,
// src/quant/int8/symmetric.rs:42-57), per tensor or per row.
//
// Two passes: an absmax reduction (order-independent, so the scale is
// bit-identical to the reference's sequential fold) and the element-wise
// quantization.  Per tensor they run in one launch with a grid barrier
// between them when the caller provides the barrier words (the values of the
// first pass mostly stay in registers: 4 B read + 1 B written per element),
// else as two kernels.  HBM-bound.
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "internal.h"

namespace mri {
namespace {

constexpr int kQThreads = 256;

// Programmatic dependent launch: the successor (typically the GEMM, which
// prefetches its weight tiles before waiting) may start now; this kernel reads
// its input only after the predecessor has completed.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t qlaunch(const DeviceInfo& dev, void (*k)(KArgs...), unsigned grid, cudaStream_t st,
                    Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dev.opt.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// Per-tensor, pass 1: every block folds its grid-stride share and writes its
// partial maximum to partial[blockIdx.x] (no atomics, no clearing needed).
__global__ void __launch_bounds__(kQThreads) absmax_tensor_kernel(const float* __restrict__ x,
                                                                  size_t n, float* partial) {
  pdl_enter();
  float m = 0.0f;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const size_t n4 = n / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    constexpr int U = 4;  // independent loads in flight per thread
    size_t j = i;
    for (; j + (U - 1) * stride < n4; j += U * stride) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = ld_act(x4 + j + u * stride);
#pragma unroll
      for (int u = 0; u < U; ++u)
        m = absmax_acc(absmax_acc(absmax_acc(absmax_acc(m, v[u].x), v[u].y), v[u].z), v[u].w);
    }
    for (; j < n4; j += stride) {
      const float4 v = ld_act(x4 + j);
      m = absmax_acc(absmax_acc(absmax_acc(absmax_acc(m, v.x), v.y), v.z), v.w);
    }
    for (size_t j = n4 * 4 + i; j < n; j += stride) m = absmax_acc(m, ld_act(x + j));
  } else {
    for (size_t j = i; j < n; j += stride) m = absmax_acc(m, ld_act(x + j));
  }
  m = warp_max(m);
  __shared__ float red[kQThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kQThreads / 32 ? red[threadIdx.x] : 0.0f;
    v = warp_max(v);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
  }
}

// Max over the `count` partial maxima, computed by every block of pass 2.
__device__ float reduce_partials(const float* __restrict__ partial, int count) {
  __shared__ float red[kQThreads / 32];
  __shared__ float result;
  float m = 0.0f;
  for (int i = threadIdx.x; i < count; i += kQThreads) m = fmaxf(m, ld_act(partial + i));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kQThreads / 32 ? red[threadIdx.x] : 0.0f;
    v = warp_max(v);
    if (threadIdx.x == 0) result = v;
  }
  __syncthreads();
  return result;
}

// Per-row: one block per row.
__global__ void __launch_bounds__(kQThreads) absmax_row_kernel(const float* __restrict__ x,
                                                               size_t k, float* amax) {
  pdl_enter();
  const float* row = x + static_cast<size_t>(blockIdx.x) * k;
  float m = 0.0f;
  for (size_t j = threadIdx.x; j < k; j += kQThreads) m = absmax_acc(m, ld_act(row + j));
  m = warp_max(m);
  __shared__ float red[kQThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kQThreads / 32 ? red[threadIdx.x] : 0.0f;
    v = warp_max(v);
    if (threadIdx.x == 0) amax[blockIdx.x] = v;
  }
}

__global__ void __launch_bounds__(kQThreads) quant_apply_kernel(const float* __restrict__ x,
                                                                size_t m, size_t k, int per_row,
                                                                const float* __restrict__ amax,
                                                                int n_partials,
                                                                int8_t* __restrict__ q,
                                                                float* __restrict__ scale_out) {
  pdl_enter();
  const size_t n = m * k;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (!per_row) {
    const float scale = sym_scale(reduce_partials(amax, n_partials));
    const float inv = __fdiv_rn(1.0f, scale);
    if (tid == 0) scale_out[0] = scale;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(q) & 3) == 0) {
      const size_t n4 = n / 4;
      const float4* x4 = reinterpret_cast<const float4*>(x);
      char4* q4 = reinterpret_cast<char4*>(q);
      constexpr int U = 4;  // independent loads in flight per thread
      size_t j = tid;
      for (; j + (U - 1) * stride < n4; j += U * stride) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = ld_act(x4 + j + u * stride);
#pragma unroll
        for (int u = 0; u < U; ++u)
          q4[j + u * stride] = make_char4(sym_quant(v[u].x, inv), sym_quant(v[u].y, inv),
                                          sym_quant(v[u].z, inv), sym_quant(v[u].w, inv));
      }
      for (; j < n4; j += stride) {
        const float4 v = ld_act(x4 + j);
        q4[j] = make_char4(sym_quant(v.x, inv), sym_quant(v.y, inv), sym_quant(v.z, inv),
                           sym_quant(v.w, inv));
      }
      for (size_t j = n4 * 4 + tid; j < n; j += stride) q[j] = sym_quant(ld_act(x + j), inv);
    } else {
      for (size_t j = tid; j < n; j += stride) q[j] = sym_quant(ld_act(x + j), inv);
    }
  } else {
    for (size_t r = tid; r < m; r += stride) scale_out[r] = sym_scale(ld_act(amax + r));
    for (size_t j = tid; j < n; j += stride) {
      const size_t r = j / k;
      const float scale = sym_scale(ld_act(amax + r));
      q[j] = sym_quant(ld_act(x + j), __fdiv_rn(1.0f, scale));
    }
  }
}

// Per row in one pass, for rows of at most kRowVec float4 per thread: block r
// reads row r once into registers, reduces its absmax and writes the
// quantized row and its scale (symmetric.rs:41-56 per row).  x and q 16- and
// 4-byte aligned, k % 4 == 0 (the launcher checks).
constexpr int kRowVec = 8;

__global__ void __launch_bounds__(kQThreads) quant_rows_kernel(const float* __restrict__ x, size_t k,
                                                               int8_t* __restrict__ q,
                                                               float* __restrict__ scale_out) {
  pdl_enter();
  const size_t k4 = k / 4;
  const float4* row = reinterpret_cast<const float4*>(x + static_cast<size_t>(blockIdx.x) * k);
  float4 v[kRowVec];
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < kRowVec; ++j) {
    const size_t i = threadIdx.x + static_cast<size_t>(j) * kQThreads;
    v[j] = i < k4 ? ld_act(row + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < kRowVec; ++j)
    m = absmax_acc(absmax_acc(absmax_acc(absmax_acc(m, v[j].x), v[j].y), v[j].z), v[j].w);
  m = warp_max(m);
  __shared__ float red[kQThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < kQThreads / 32; ++i) t = fmaxf(t, red[i]);
  const float scale = sym_scale(t);
  const float inv = __fdiv_rn(1.0f, scale);
  if (threadIdx.x == 0) scale_out[blockIdx.x] = scale;
  char4* qr = reinterpret_cast<char4*>(q + static_cast<size_t>(blockIdx.x) * k);
#pragma unroll
  for (int j = 0; j < kRowVec; ++j) {
    const size_t i = threadIdx.x + static_cast<size_t>(j) * kQThreads;
    if (i < k4) {
      char4 o;
      o.x = sym_quant(v[j].x, inv);
      o.y = sym_quant(v[j].y, inv);
      o.z = sym_quant(v[j].z, inv);
      o.w = sym_quant(v[j].w, inv);
      qr[i] = o;
    }
  }
}

// Fused producer ops (RMSNorm or SwiGLU) in front of the quantizer.  Pass 1,
// one block per row: 1/rms of the row (RMSNorm) into row_inv[r] and the
// absmax of the row's transformed values into partial[r].
__device__ __forceinline__ float xform(const float* __restrict__ x, size_t k, size_t K, int r,
                                       const float* __restrict__ norm_w, float inv_r, int swiglu) {
  if (swiglu) {
    const float g = ld_act(x + static_cast<size_t>(r) * 2 * K + 2 * k);
    const float u = ld_act(x + static_cast<size_t>(r) * 2 * K + 2 * k + 1);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
  }
  const float v = ld_act(x + static_cast<size_t>(r) * K + k);
  return norm_w ? __fmul_rn(__ldg(norm_w + k), __fmul_rn(v, inv_r)) : v;
}

// Four transformed elements k..k+3 of row r (K % 4 == 0, 16-byte aligned x
// and norm_w): the same arithmetic as xform, element by element.
__device__ __forceinline__ float4 xform4(const float* __restrict__ x, size_t k, size_t K, int r,
                                         const float* __restrict__ norm_w, float inv_r, int swiglu) {
  if (swiglu) {
    const float* row = x + static_cast<size_t>(r) * 2 * K + 2 * k;
    const float4 a = ld_act(reinterpret_cast<const float4*>(row));
    const float4 b = ld_act(reinterpret_cast<const float4*>(row + 4));
    return make_float4(__fmul_rn(__fdiv_rn(a.x, __fadd_rn(1.0f, expf(-a.x))), a.y),
                       __fmul_rn(__fdiv_rn(a.z, __fadd_rn(1.0f, expf(-a.z))), a.w),
                       __fmul_rn(__fdiv_rn(b.x, __fadd_rn(1.0f, expf(-b.x))), b.y),
                       __fmul_rn(__fdiv_rn(b.z, __fadd_rn(1.0f, expf(-b.z))), b.w));
  }
  float4 v = ld_act(reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * K + k));
  if (norm_w) {
    const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w + k));
    v = make_float4(__fmul_rn(w.x, __fmul_rn(v.x, inv_r)), __fmul_rn(w.y, __fmul_rn(v.y, inv_r)),
                    __fmul_rn(w.z, __fmul_rn(v.z, inv_r)), __fmul_rn(w.w, __fmul_rn(v.w, inv_r)));
  }
  return v;
}

__global__ void __launch_bounds__(kQThreads) row_stats_kernel(const float* __restrict__ x, size_t K,
                                                              const float* __restrict__ norm_w,
                                                              float eps, int swiglu,
                                                              float* __restrict__ row_inv,
                                                              float* __restrict__ partial) {
  pdl_enter();
  const int r = blockIdx.x;
  __shared__ float red[kQThreads / 32];
  __shared__ float inv_s;
  float inv_r = 1.0f;
  // float4 loads, four in flight per thread, when rows allow it.
  const bool vec = K % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (!norm_w || (reinterpret_cast<uintptr_t>(norm_w) & 15) == 0);
  if (norm_w) {
    float ss = 0.0f;
    if (vec) {
      const float4* row = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * K);
      const size_t k4 = K / 4;
      for (size_t i0 = threadIdx.x; i0 < k4; i0 += 4 * kQThreads) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          v[u] = i0 + u * kQThreads < k4 ? ld_act(row + i0 + u * kQThreads) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          ss = __fmaf_rn(v[u].x, v[u].x, ss);
          ss = __fmaf_rn(v[u].y, v[u].y, ss);
          ss = __fmaf_rn(v[u].z, v[u].z, ss);
          ss = __fmaf_rn(v[u].w, v[u].w, ss);
        }
      }
    } else
    for (size_t k = threadIdx.x; k < K; k += kQThreads) {
      const float v = ld_act(x + static_cast<size_t>(r) * K + k);
      ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum_f(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      for (int i = 0; i < kQThreads / 32; ++i) t += red[i];
      inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, static_cast<float>(K)), eps)));
      row_inv[r] = inv_s;
    }
    __syncthreads();
    inv_r = inv_s;
  }
  float m = 0.0f;
  if (vec) {
    const size_t k4 = K / 4;
    for (size_t i0 = threadIdx.x; i0 < k4; i0 += 4 * kQThreads) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        v[u] = i0 + u * kQThreads < k4 ? xform4(x, (i0 + u * kQThreads) * 4, K, r, norm_w, inv_r, swiglu)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        m = absmax_acc(absmax_acc(absmax_acc(absmax_acc(m, v[u].x), v[u].y), v[u].z), v[u].w);
    }
  } else {
    for (size_t k = threadIdx.x; k < K; k += kQThreads) m = absmax_acc(m, xform(x, k, K, r, norm_w, inv_r, swiglu));
  }
  m = warp_max(m);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < kQThreads / 32; ++i) t = fmaxf(t, red[i]);
    partial[r] = t;
  }
}

// Pass 2: per-tensor (or per-row) scale from the row maxima, quantize the
// transformed values.
__global__ void __launch_bounds__(kQThreads) quant_apply_xform_kernel(
    const float* __restrict__ x, size_t m, size_t K, int per_row, const float* __restrict__ partial,
    const float* __restrict__ norm_w, const float* __restrict__ row_inv, int swiglu,
    int8_t* __restrict__ q, float* __restrict__ scale_out) {
  pdl_enter();
  const size_t n = m * K;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  float inv_t = 0.0f;
  if (!per_row) {
    const float scale = sym_scale(reduce_partials(partial, static_cast<int>(m)));
    inv_t = __fdiv_rn(1.0f, scale);
    if (tid == 0) scale_out[0] = scale;
  } else {
    for (size_t r = tid; r < m; r += stride) scale_out[r] = sym_scale(ld_act(partial + r));
  }
  const bool vec = K % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (!norm_w || (reinterpret_cast<uintptr_t>(norm_w) & 15) == 0) &&
                   (reinterpret_cast<uintptr_t>(q) & 3) == 0;
  if (vec) {
    // Four elements of one row per step (K % 4 == 0).
    const size_t K4 = K / 4;
    for (size_t j = tid; j < n / 4; j += stride) {
      const int r = static_cast<int>(j / K4);
      const size_t k = (j - r * K4) * 4;
      const float inv = per_row ? __fdiv_rn(1.0f, sym_scale(ld_act(partial + r))) : inv_t;
      float4 v;
      if (swiglu) {
        const float* row = x + static_cast<size_t>(r) * 2 * K + 2 * k;
        const float4 a = ld_act(reinterpret_cast<const float4*>(row));
        const float4 b = ld_act(reinterpret_cast<const float4*>(row + 4));
        v.x = __fmul_rn(__fdiv_rn(a.x, __fadd_rn(1.0f, expf(-a.x))), a.y);
        v.y = __fmul_rn(__fdiv_rn(a.z, __fadd_rn(1.0f, expf(-a.z))), a.w);
        v.z = __fmul_rn(__fdiv_rn(b.x, __fadd_rn(1.0f, expf(-b.x))), b.y);
        v.w = __fmul_rn(__fdiv_rn(b.z, __fadd_rn(1.0f, expf(-b.z))), b.w);
      } else {
        v = ld_act(reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * K + k));
        if (norm_w) {
          const float ir = ld_act(row_inv + r);
          const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w + k));
          v.x = __fmul_rn(w.x, __fmul_rn(v.x, ir));
          v.y = __fmul_rn(w.y, __fmul_rn(v.y, ir));
          v.z = __fmul_rn(w.z, __fmul_rn(v.z, ir));
          v.w = __fmul_rn(w.w, __fmul_rn(v.w, ir));
        }
      }
      char4 o;
      o.x = sym_quant(v.x, inv);
      o.y = sym_quant(v.y, inv);
      o.z = sym_quant(v.z, inv);
      o.w = sym_quant(v.w, inv);
      reinterpret_cast<char4*>(q)[j] = o;
    }
    return;
  }
  for (size_t j = tid; j < n; j += stride) {
    const int r = static_cast<int>(j / K);
    const size_t k = j % K;
    const float inv = per_row ? __fdiv_rn(1.0f, sym_scale(ld_act(partial + r))) : inv_t;
    q[j] = sym_quant(xform(x, k, K, r, norm_w, norm_w ? ld_act(row_inv + r) : 1.0f, swiglu), inv);
  }
}

// ── one-launch per-tensor quantizers ─────────────────────────────────────────
// Both passes in one kernel: every block folds its share into a partial
// maximum, the blocks meet at a grid barrier (sense reversal on sync[0] =
// arrivals, sync[1] = generation; the last block to arrive reduces the
// partials, publishes the scale, resets the count and advances the
// generation), then each block quantizes its share, from registers where it
// kept the values.  The result is bit-identical to the two-kernel path (the
// same partial maxima, scale and element arithmetic).  The grid never exceeds
// the blocks that fit on the device at once.  Every block releases the
// successor kernel (griddepcontrol.launch_dependents) as it starts: the
// successor can only launch once every block of this grid has done so, i.e.
// once the whole grid is resident, so its CTAs cannot keep a block of this
// grid from starting, and it prefetches its weights while this kernel runs.
// The wait is bounded: on timeout the kernel records MRI_ERR_TIMEOUT and
// returns without writing the output.
constexpr int kOnceCache = 4;  // float4 per thread kept between the passes (flat kernel)

__device__ __forceinline__ float absmax4(float m, float4 v) {
  return absmax_acc(absmax_acc(absmax_acc(absmax_acc(m, v.x), v.y), v.z), v.w);
}

__device__ __forceinline__ char4 quant4(float4 v, float inv) {
  return make_char4(sym_quant(v.x, inv), sym_quant(v.y, inv), sym_quant(v.z, inv), sym_quant(v.w, inv));
}

// Grid barrier of the one-launch quantizers.  With write_partial, the block's
// maximum of the per-thread values `m` is first written to
// partial[blockIdx.x]; the last block to arrive reduces partial[0,
// n_partials).  Returns the tensor's scale in every thread, or -1 after a
// timeout.
__device__ float once_barrier_scale(float m, bool write_partial, float* __restrict__ partial, int n_partials,
                                    unsigned* sync, float* __restrict__ scale_out, int* status) {
  __shared__ float red[kQThreads / 32];
  __shared__ float s_scale;
  __shared__ int s_last;
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  unsigned gen0 = 0;
  if (threadIdx.x == 0) {
    if (write_partial) {
      float t = 0.0f;
#pragma unroll
      for (int i = 0; i < kQThreads / 32; ++i) t = fmaxf(t, red[i]);
      partial[blockIdx.x] = t;
    }
    gen0 = *reinterpret_cast<volatile unsigned*>(sync + 1);
    __threadfence();
    s_last = atomicAdd(sync, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    float t = 0.0f;
    for (int i = threadIdx.x; i < n_partials; i += kQThreads) t = fmaxf(t, __ldcg(partial + i));
    t = warp_max(t);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = 0.0f;
#pragma unroll
      for (int i = 0; i < kQThreads / 32; ++i) v = fmaxf(v, red[i]);
      const float scale = sym_scale(v);
      scale_out[0] = scale;
      s_scale = scale;
      sync[0] = 0;
      __threadfence();
      atomicAdd(sync + 1, 1u);
    }
  } else if (threadIdx.x == 0) {
    const long long t0 = clock64();
    float scale = 0.0f;
    for (;;) {
      if (*reinterpret_cast<volatile unsigned*>(sync + 1) != gen0) {
        __threadfence();
        scale = __ldcg(scale_out);
        break;
      }
      if (clock64() - t0 > kWaitBudgetClocks) {
        if (status) *reinterpret_cast<volatile int*>(status) = MRI_ERR_TIMEOUT;
        scale = -1.0f;
        break;
      }
      __nanosleep(20);
    }
    s_scale = scale;
  }
  __syncthreads();
  return s_scale;
}

// Flat: a grid-stride share of the n4 float4 of x (16-byte aligned, q 4-byte
// aligned); the first kOnceCache of each thread stay in registers.
__global__ void __launch_bounds__(kQThreads) quant_tensor_once_kernel(const float* __restrict__ x, size_t n4,
                                                                      float* __restrict__ partial,
                                                                      unsigned* sync,
                                                                      int8_t* __restrict__ q,
                                                                      float* __restrict__ scale_out,
                                                                      int* status) {
  pdl_enter();
  const float4* x4 = reinterpret_cast<const float4*>(x);
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  float4 v[kOnceCache];
  float m = 0.0f;
#pragma unroll
  for (int u = 0; u < kOnceCache; ++u) {
    const size_t j = tid + u * stride;
    v[u] = j < n4 ? ld_act(x4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int u = 0; u < kOnceCache; ++u) m = absmax4(m, v[u]);
  size_t j = tid + kOnceCache * stride;
  for (; j + 3 * stride < n4; j += 4 * stride) {
    float4 w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w[u] = ld_act(x4 + j + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) m = absmax4(m, w[u]);
  }
  for (; j < n4; j += stride) m = absmax4(m, ld_act(x4 + j));
  const float scale = once_barrier_scale(m, true, partial, gridDim.x, sync, scale_out, status);
  if (scale < 0.0f) return;
  const float inv = __fdiv_rn(1.0f, scale);
  char4* q4 = reinterpret_cast<char4*>(q);
#pragma unroll
  for (int u = 0; u < kOnceCache; ++u) {
    const size_t i = tid + u * stride;
    if (i < n4) q4[i] = quant4(v[u], inv);
  }
  for (j = tid + kOnceCache * stride; j < n4; j += stride) q4[j] = quant4(ld_act(x4 + j), inv);
}

// Row-wise, with the producer op fused in front (RMSNorm with weight norm_w,
// or SwiGLU over interleaved gate/up rows of width 2K): block b takes rows b,
// b + grid, ...; a row's transformed values are formed once per pass from its
// K / 4 float4 (thread t: float4 t, t + 256, ..., at most kVec), its 1/rms
// and maximum go to row_inv[r] and partial[r], and the block's first row
// stays in registers.  The same arithmetic, in the same order, as
// row_stats_kernel + quant_apply_xform_kernel.  per_row: each row's own scale
// (no barrier).  K % 4 == 0, x / norm_w 16-byte aligned, q 4-byte aligned.
template <int kVec>
__device__ __forceinline__ void load_xform_row(const float* __restrict__ x, size_t K, int r,
                                               const float* __restrict__ norm_w, float eps, int swiglu,
                                               float4 (&v)[kVec], float* inv_out) {
  const size_t k4 = K / 4;
  __shared__ float red[kQThreads / 32];
  __shared__ float inv_s;
  if (swiglu) {
    const float4* row = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * 2 * K);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const size_t i = threadIdx.x + static_cast<size_t>(j) * kQThreads;
      if (i < k4) {
        const float4 a = ld_act(row + 2 * i), b = ld_act(row + 2 * i + 1);
        v[j] = make_float4(__fmul_rn(__fdiv_rn(a.x, __fadd_rn(1.0f, expf(-a.x))), a.y),
                           __fmul_rn(__fdiv_rn(a.z, __fadd_rn(1.0f, expf(-a.z))), a.w),
                           __fmul_rn(__fdiv_rn(b.x, __fadd_rn(1.0f, expf(-b.x))), b.y),
                           __fmul_rn(__fdiv_rn(b.z, __fadd_rn(1.0f, expf(-b.z))), b.w));
      } else {
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    *inv_out = 1.0f;
    return;
  }
  const float4* row = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * K);
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const size_t i = threadIdx.x + static_cast<size_t>(j) * kQThreads;
    v[j] = i < k4 ? ld_act(row + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (!norm_w) {
    *inv_out = 1.0f;
    return;
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    ss = __fmaf_rn(v[j].x, v[j].x, ss);
    ss = __fmaf_rn(v[j].y, v[j].y, ss);
    ss = __fmaf_rn(v[j].z, v[j].z, ss);
    ss = __fmaf_rn(v[j].w, v[j].w, ss);
  }
  ss = warp_sum_f(ss);
  __syncthreads();  // red / inv_s of the previous row are no longer read
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < kQThreads / 32; ++i) t += red[i];
    inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, static_cast<float>(K)), eps)));
  }
  __syncthreads();
  const float ir = inv_s;
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const size_t i = threadIdx.x + static_cast<size_t>(j) * kQThreads;
    if (i < k4) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w) + i);
      v[j] = make_float4(__fmul_rn(w.x, __fmul_rn(v[j].x, ir)), __fmul_rn(w.y, __fmul_rn(v[j].y, ir)),
                         __fmul_rn(w.z, __fmul_rn(v[j].z, ir)), __fmul_rn(w.w, __fmul_rn(v[j].w, ir)));
    }
  }
  *inv_out = ir;
}

template <int kVec>
__device__ __forceinline__ float row_block_max(const float4 (&v)[kVec]) {
  __shared__ float red[kQThreads / 32];
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < kVec; ++j) m = absmax4(m, v[j]);
  m = warp_max(m);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < kQThreads / 32; ++i) t = fmaxf(t, red[i]);
  return t;
}

template <int kVec>
__device__ __forceinline__ void store_row_q(const float4 (&v)[kVec], size_t K, int r, float inv,
                                            int8_t* __restrict__ q) {
  const size_t k4 = K / 4;
  char4* qr = reinterpret_cast<char4*>(q + static_cast<size_t>(r) * K);
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const size_t i = threadIdx.x + static_cast<size_t>(j) * kQThreads;
    if (i < k4) qr[i] = quant4(v[j], inv);
  }
}

template <int kVec>
__global__ void __launch_bounds__(kQThreads) quant_rows_once_kernel(
    const float* __restrict__ x, int m, size_t K, const float* __restrict__ norm_w, float eps, int swiglu,
    int per_row, float* __restrict__ partial, unsigned* sync, int8_t* __restrict__ q,
    float* __restrict__ scale_out, int* status) {
  pdl_enter();
  float4 v[kVec];
  float ir0 = 1.0f;
  const int r0 = blockIdx.x;
  // Pass 1.  The block's first row stays in v.
  load_xform_row<kVec>(x, K, r0, norm_w, eps, swiglu, v, &ir0);
  float mx = row_block_max<kVec>(v);
  if (threadIdx.x == 0) partial[r0] = mx;
  if (per_row) {
    if (threadIdx.x == 0) scale_out[r0] = sym_scale(mx);
    store_row_q<kVec>(v, K, r0, __fdiv_rn(1.0f, sym_scale(mx)), q);
    for (int r = r0 + gridDim.x; r < m; r += gridDim.x) {
      float ir;
      load_xform_row<kVec>(x, K, r, norm_w, eps, swiglu, v, &ir);
      const float t = row_block_max<kVec>(v);
      if (threadIdx.x == 0) scale_out[r] = sym_scale(t);
      store_row_q<kVec>(v, K, r, __fdiv_rn(1.0f, sym_scale(t)), q);
    }
    return;
  }
  float4 w[kVec];
  for (int r = r0 + gridDim.x; r < m; r += gridDim.x) {
    float ir;
    load_xform_row<kVec>(x, K, r, norm_w, eps, swiglu, w, &ir);
    const float t = row_block_max<kVec>(w);
    if (threadIdx.x == 0) partial[r] = t;
  }
  const float scale = once_barrier_scale(0.0f, false, partial, m, sync, scale_out, status);
  if (scale < 0.0f) return;
  const float inv = __fdiv_rn(1.0f, scale);
  store_row_q<kVec>(v, K, r0, inv, q);
  for (int r = r0 + gridDim.x; r < m; r += gridDim.x) {
    float ir;
    load_xform_row<kVec>(x, K, r, norm_w, eps, swiglu, w, &ir);
    store_row_q<kVec>(w, K, r, inv, q);
  }
}

// Result rows from device memory into a caller's pinned host buffer (mapped
// into the device's address space), 16 bytes per store, after the producing
// kernel has finished.
__global__ void __launch_bounds__(kQThreads) copy_out_kernel(const float4* __restrict__ src,
                                                             float4* __restrict__ dst, size_t n4) {
  pdl_enter();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = ld_act(src + i);
}

__global__ void add_inplace_kernel(float* __restrict__ out, const float* __restrict__ res, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = __fadd_rn(res[i], out[i]);
}

}  // namespace

cudaError_t launch_copy_out(const DeviceInfo& dev, cudaStream_t st, const float* src, float* dst,
                            size_t n, LaunchStats* ls) {
  if (n % 4 != 0 || (reinterpret_cast<uintptr_t>(src) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(dst) & 15) != 0)
    return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const size_t n4 = n / 4;
  const unsigned grid = static_cast<unsigned>(std::min<size_t>(dev.sm_count, (n4 + kQThreads - 1) / kQThreads));
  cudaError_t e = qlaunch(dev, copy_out_kernel, grid, st, reinterpret_cast<const float4*>(src),
                          reinterpret_cast<float4*>(dst), n4);
  if (ls) ls->launches++;
  return e;
}

cudaError_t launch_add_residual(const DeviceInfo& dev, cudaStream_t st, float* out,
                                const float* residual, size_t n, LaunchStats* ls) {
  const int blocks = static_cast<int>(std::max<size_t>(1, std::min<size_t>(dev.sm_count * 8, (n + 255) / 256)));
  add_inplace_kernel<<<blocks, 256, 0, st>>>(out, residual, n);
  if (ls) ls->launches++;
  return cudaGetLastError();
}

// Blocks of `k` that fit on one SM, cached per kernel and device.
template <typename KernelT>
int once_resident(KernelT k, int device) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(reinterpret_cast<const void*>(k), device);
  auto it = done.find(key);
  if (it != done.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kQThreads, 0) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  done[key] = n;
  return n;
}

cudaError_t launch_quantize(const DeviceInfo& dev, cudaStream_t st, const float* x, size_t m,
                            size_t k, int per_row, int8_t* q, float* scale, float* amax_scratch,
                            LaunchStats* ls, const float* norm_w, float eps, int swiglu,
                            unsigned* sync, int* status) {
  const size_t n = m * k;
  const bool x16 = (reinterpret_cast<uintptr_t>(x) & 15) == 0, q4 = (reinterpret_cast<uintptr_t>(q) & 3) == 0;
  if ((norm_w || swiglu) && n > 0) {
    // amax_scratch holds 2 * max(m, kQuantPartials) floats: row maxima, then 1/rms.
    float* partial = amax_scratch;
    float* row_inv = amax_scratch + std::max(m, kQuantPartials);
    const size_t k4 = k / 4;
    const bool once = (sync || per_row) && k % 4 == 0 && x16 && q4 &&
                      (!norm_w || (reinterpret_cast<uintptr_t>(norm_w) & 15) == 0) &&
                      k4 <= 12 * static_cast<size_t>(kQThreads) && m <= (1u << 30);
    if (once) {
      const bool small = k4 <= 4 * static_cast<size_t>(kQThreads);
      auto kern = small ? quant_rows_once_kernel<4> : quant_rows_once_kernel<12>;
      // Only when every row gets a block of its own (a block that took a
      // second row would read and transform it twice).
      const int fit = once_resident(kern, dev.device) * dev.sm_count;
      if (fit > 0 && m <= static_cast<size_t>(fit)) {
        const unsigned grid = static_cast<unsigned>(m);
        cudaError_t e = qlaunch(dev, kern, grid, st, x, static_cast<int>(m), k, norm_w, eps, swiglu, per_row,
                                partial, sync, q, scale, status);
        if (ls) ls->launches++;
        return e;
      }
    }
    cudaError_t e = qlaunch(dev, row_stats_kernel, static_cast<unsigned>(m), st, x, k, norm_w, eps, swiglu,
                            row_inv, partial);
    if (e != cudaSuccess) return e;
    const int apply_blocks = static_cast<int>(std::max<size_t>(
        1, std::min<size_t>(static_cast<size_t>(dev.sm_count) * 8, (n + kQThreads * 4 - 1) / (kQThreads * 4))));
    e = qlaunch(dev, quant_apply_xform_kernel, static_cast<unsigned>(apply_blocks), st, x, m, k, per_row,
                partial, norm_w, row_inv, swiglu, q, scale);
    if (ls) ls->launches += 2;
    return e;
  }
  if (n == 0) {
    // Empty input: the reference's fold yields 0 -> scale 1.0.
    if (!per_row) {
      const float one = 1.0f;
      return cudaMemcpyAsync(scale, &one, sizeof(float), cudaMemcpyHostToDevice, st);
    }
    if (m == 0) return cudaSuccess;
  }
  if (per_row && k % 4 == 0 && k <= static_cast<size_t>(kRowVec) * kQThreads * 4 && x16 && q4) {
    cudaError_t e = qlaunch(dev, quant_rows_kernel, static_cast<unsigned>(m), st, x, k, q, scale);
    if (ls) ls->launches++;
    return e;
  }
  if (!per_row && sync && n % 4 == 0 && x16 && q4) {
    const int fit = once_resident(quant_tensor_once_kernel, dev.device) * dev.sm_count;
    if (fit > 0) {
      const size_t n4 = n / 4;
      const unsigned grid = static_cast<unsigned>(std::max<size_t>(
          1, std::min<size_t>(std::min<size_t>(std::min<size_t>(static_cast<size_t>(fit), 4 * dev.sm_count),
                                               kQuantPartials),
                              (n4 + kQThreads - 1) / kQThreads)));
      cudaError_t e = qlaunch(dev, quant_tensor_once_kernel, grid, st, x, n4, amax_scratch, sync, q, scale, status);
      if (ls) ls->launches++;
      return e;
    }
  }
  // Pass 1 writes one partial maximum per block into amax_scratch, which must
  // hold kQuantPartials floats (per tensor) or m floats (per row).
  const int blocks = static_cast<int>(std::max<size_t>(
      1, std::min<size_t>(std::min<size_t>(static_cast<size_t>(dev.sm_count) * 2, kQuantPartials),
                          (n + kQThreads * 16 - 1) / (kQThreads * 16))));
  cudaError_t e = per_row
                      ? qlaunch(dev, absmax_row_kernel, static_cast<unsigned>(m), st, x, k, amax_scratch)
                      : qlaunch(dev, absmax_tensor_kernel, static_cast<unsigned>(blocks), st, x, n, amax_scratch);
  if (e != cudaSuccess) return e;
  if (ls) ls->launches++;
  const int apply_blocks = static_cast<int>(std::max<size_t>(
      1, std::min<size_t>(static_cast<size_t>(dev.sm_count) * 8, (n + kQThreads * 4 - 1) / (kQThreads * 4))));
  e = qlaunch(dev, quant_apply_kernel, static_cast<unsigned>(apply_blocks), st, x, m, k, per_row,
              amax_scratch, blocks, q, scale);
  if (ls) ls->launches++;
  return e;
}

}  // namespace mri
