// gemv.cu — K2/K4/K5: memory-bound products for M <= 8 activation rows.
//
// Shape of every "stream" kernel (one CTA per SM, persistent over a balanced,
// contiguous range of weight rows):
//   warp 0, lane 0 : producer.  Streams 8-row groups of the weight matrix
//                    into a ring of shared-memory stages with 1-D bulk TMA
//                    copies (cp.async.bulk, L2 evict-first), one mbarrier
//                    "full" per stage, waiting on "empty" before reuse.
//   warps 1..8     : consumers.  Warp w owns row w of each stage; its lanes
//                    split the row's K bytes, the activations sit in shared
//                    memory (quantized once per CTA in the prologue, which
//                    overlaps the first weight copies), and the epilogue
//                    rescales to f32.
// Every wait is bounded (mbar_wait); on timeout the kernel records
// MRI_ERR_TIMEOUT in the context status word and returns.
//
// Bit-exactness: INT8 products sum integers (order-free) and apply the
// reference epilogue `(f32)acc * s_a * s_w`; Q8_0 computes each block term
// `(f32)dot * s_a * d` and adds the terms in block order on one lane, as
// q8_direct.rs:266-285 does.  Q4_0 reassociates its f32 sum (tolerance).
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include <cuda_bf16.h>

#include "common.cuh"
#include "internal.h"

namespace mri {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kRowsPerStage = kConsumerWarps;
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kMaxStages = 6;
constexpr size_t kSmemBudget = 220 * 1024;  // of the 227 KB opt-in per CTA

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Programmatic dependent launch: the next kernel in the stream may start as
// soon as every CTA of this one has passed pdl_launch_dependents(); it must
// call pdl_wait() before touching anything this kernel writes.  Weights are
// constant, so producers stream them before pdl_wait(); activations are read
// and outputs written only after it.  Both are no-ops without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Shared-memory layout of a stream kernel.
struct StreamLayout {
  size_t bars;       // 2 * stages mbarriers
  size_t scales;     // 8 activation scales + 8 reduction slots
  size_t act;        // activation buffer
  size_t extra;      // per-warp scratch (Q8_0 term buffer)
  size_t stage;      // first stage buffer
  size_t stage_bytes;
  size_t total;
  int stages;
};

__host__ __device__ inline StreamLayout make_layout(size_t act_bytes, size_t extra_bytes,
                                                    size_t stage_bytes, int stages) {
  StreamLayout L{};
  L.stages = stages;
  L.bars = 0;
  L.scales = align_up((2 * stages + 2) * sizeof(uint64_t), 16);  // + act-issued barrier
  L.act = align_up(L.scales + 16 * sizeof(float), 128);
  L.extra = align_up(L.act + act_bytes, 128);
  L.stage = align_up(L.extra + extra_bytes, 128);
  L.stage_bytes = align_up(stage_bytes, 128);
  // 16 bytes of slack: block loaders read whole words and may pass the end
  // of the last row by up to 2 bytes.
  L.total = L.stage + L.stage_bytes * stages + 16;
  return L;
}

// Rows [begin, end) of this CTA: a balanced split of N in units of `gran` rows.
__device__ __forceinline__ void cta_rows(size_t N, size_t gran, size_t& begin, size_t& end) {
  const size_t units = (N + gran - 1) / gran;
  const size_t u0 = units * blockIdx.x / gridDim.x;
  const size_t u1 = units * (blockIdx.x + 1) / gridDim.x;
  begin = u0 * gran;
  end = std::min(N, u1 * gran);
}

// Producer loop shared by all stream kernels: stage `it` holds rows
// [begin + 8*it, ...) whose bytes start at W + row*row_bytes.
__device__ void stream_producer(const uint8_t* W, size_t row_bytes, size_t begin, size_t end,
                                uint64_t* full, uint64_t* empty, uint8_t* stages_base,
                                size_t stage_stride, int n_stages, int* status,
                                uint64_t* act_issued = nullptr, int pre = 1 << 30) {
  const uint64_t policy = l2_policy_evict_first();
  const int iters = static_cast<int>((end - begin + kRowsPerStage - 1) / kRowsPerStage);
  int issued = 0;
  for (int it = 0; it < iters; ++it) {
    const int s = it % n_stages;
    // Stages after the first `pre` wait until the activation loads are issued.
    if (act_issued && it == pre && !mbar_wait(act_issued, 0, status)) break;
    if (it >= n_stages) {
      if (!mbar_wait(&empty[s], ((it / n_stages) - 1) & 1, status)) break;
    }
    const size_t r0 = begin + static_cast<size_t>(it) * kRowsPerStage;
    const size_t nrows = std::min<size_t>(kRowsPerStage, end - r0);
    const uint32_t bytes = static_cast<uint32_t>(align_up(nrows * row_bytes, 16));
    mbar_arrive_expect_tx(&full[s], bytes);
    bulk_copy_g2s_stream(stages_base + s * stage_stride, W + r0 * row_bytes, bytes, &full[s],
                         policy);
    issued = it + 1;
  }
  // Drain: return only once every copy this thread issued has landed.
  for (int it = std::max(0, issued - n_stages); it < issued; ++it)
    mbar_wait(&full[it % n_stages], (it / n_stages) & 1, status);
}

__device__ __forceinline__ void init_barriers(uint64_t* full, uint64_t* empty, int n_stages,
                                              uint64_t* act_issued = nullptr) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    if (act_issued) mbar_init(act_issued, kConsumerWarps);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();
}

// ── activation prologue (consumer threads only) ──────────────────────────────

// Block-wide (consumer) max; `red` holds kConsumerWarps floats.
__device__ __forceinline__ float consumer_max(float v, float* red) {
  const int cw = (threadIdx.x >> 5) - 1;
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) red[cw] = v;
  named_bar_sync(1, kConsumerThreads);
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) r = fmaxf(r, red[i]);
  named_bar_sync(1, kConsumerThreads);
  return r;
}

__device__ __forceinline__ float consumer_sum(float v, float* red) {
  const int cw = (threadIdx.x >> 5) - 1;
  v = warp_sum_f(v);
  if ((threadIdx.x & 31) == 0) red[cw] = v;
  named_bar_sync(1, kConsumerThreads);
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) r += red[i];
  named_bar_sync(1, kConsumerThreads);
  return r;
}

// silu(g) * u (ops/activation/swiglu.rs:39-61, silu.rs:23-26).
__device__ __forceinline__ float swiglu1(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// The f32 activation element the quantizer sees: x itself, its RMSNorm
// (w[k] * (x * inv_rms[r])), or silu(gate) * up.  Four elements at a time;
// K % 4 == 0 and 16-byte aligned rows (checked by the launcher).
struct ActView {
  const float* x;
  const float* w;       // RMSNorm weight or nullptr
  const float* inv;     // per-row 1/rms (shared memory) when w != nullptr
  size_t K, ld;         // ld = K, or 2K for interleaved gate/up rows
  int swiglu;

  __device__ __forceinline__ float4 get(int r, size_t k) const {
    const float* row = x + r * ld;
    if (swiglu) {
      const float4 a = ld_act(reinterpret_cast<const float4*>(row + 2 * k));
      const float4 b = ld_act(reinterpret_cast<const float4*>(row + 2 * k + 4));
      return make_float4(swiglu1(a.x, a.y), swiglu1(a.z, a.w), swiglu1(b.x, b.y), swiglu1(b.z, b.w));
    }
    float4 v = ld_act(reinterpret_cast<const float4*>(row + k));
    if (w) v = norm(v, r, k);
    return v;
  }
  __device__ __forceinline__ float4 norm(float4 v, int r, size_t k) const {
    const float4 ww = __ldg(reinterpret_cast<const float4*>(w + k));
    const float iv = inv[r];
    return make_float4(__fmul_rn(ww.x, __fmul_rn(v.x, iv)), __fmul_rn(ww.y, __fmul_rn(v.y, iv)),
                       __fmul_rn(ww.z, __fmul_rn(v.z, iv)), __fmul_rn(ww.w, __fmul_rn(v.w, iv)));
  }
};

__device__ __forceinline__ float absmax4(float m, float4 v) {
  return absmax_acc(absmax_acc(absmax_acc(absmax_acc(m, v.x), v.y), v.z), v.w);
}

__device__ __forceinline__ char4 quant4(float4 v, float inv) {
  char4 o;
  o.x = sym_quant(v.x, inv);
  o.y = sym_quant(v.y, inv);
  o.z = sym_quant(v.z, inv);
  o.w = sym_quant(v.w, inv);
  return o;
}

// Quantize (or copy) the M activation rows into shared memory as int8 [M][K]
// row-major and fill s_scale[0..M).  Optional fused producer ops (RMSNorm,
// SwiGLU) are applied to the f32 values first.  VEC > 0 selects the decode
// path: per-tensor f32 input of at most VEC float4 per consumer thread, read
// once into registers (the host checks the preconditions).  Each consumer
// warp arrives on `act_issued` (nullable) once its activation loads are in
// flight: the producer holds back later weight stages until then, so those
// loads do not queue behind them.
template <int M, int VEC>
__device__ void load_act_i8_rowmajor(const ActArgs& act, size_t K, int8_t* s_act, float* s_scale,
                                     float* red, uint64_t* act_issued) {
  const int ct = threadIdx.x - 32;
  const size_t total = static_cast<size_t>(M) * K;
  __shared__ float s_inv[8];
  if constexpr (VEC > 0) {
    ActView v{act.x, act.norm_w, s_inv, K, K, 0};
    float4 x4[VEC];
    const int n4 = static_cast<int>(total / 4), K32 = static_cast<int>(K);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const int i = ct + j * kConsumerThreads;
      x4[j] = i < n4 ? ld_act(reinterpret_cast<const float4*>(act.x) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (act_issued) {
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(act_issued);
    }
    if (act.norm_w) {
      for (int r = 0; r < M; ++r) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const int i = ct + j * kConsumerThreads;
          if (i < n4 && (M == 1 || (i * 4) / K32 == r)) {
            ss = __fmaf_rn(x4[j].x, x4[j].x, ss);
            ss = __fmaf_rn(x4[j].y, x4[j].y, ss);
            ss = __fmaf_rn(x4[j].z, x4[j].z, ss);
            ss = __fmaf_rn(x4[j].w, x4[j].w, ss);
          }
        }
        ss = consumer_sum(ss, red);
        if (ct == 0) s_inv[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), act.eps)));
      }
      named_bar_sync(1, kConsumerThreads);
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const int i = ct + j * kConsumerThreads;
        if (i < n4) x4[j] = v.norm(x4[j], M == 1 ? 0 : (i * 4) / K32, M == 1 ? i * 4 : (i * 4) % K32);
      }
    }
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < VEC; ++j) m = absmax4(m, x4[j]);
    const float scale = sym_scale(consumer_max(m, red));
    const float inv = __fdiv_rn(1.0f, scale);
    if (ct < M) s_scale[ct] = scale;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const int i = ct + j * kConsumerThreads;
      if (i < n4) reinterpret_cast<char4*>(s_act)[i] = quant4(x4[j], inv);
    }
    named_bar_sync(1, kConsumerThreads);
    return;
  }
  if (act_issued && (threadIdx.x & 31) == 0) mbar_arrive(act_issued);
  if (act.mode == ACT_F32_PER_TENSOR || act.mode == ACT_F32_PER_ROW) {
    ActView v{act.x, act.norm_w, s_inv, K, act.swiglu ? 2 * K : K, act.swiglu};
    const bool vec = (reinterpret_cast<uintptr_t>(act.x) & 15) == 0 && K % 4 == 0 &&
                     (!act.norm_w || (reinterpret_cast<uintptr_t>(act.norm_w) & 15) == 0);
    if (false) {
    } else if (vec) {
      // Rows of K/4 float4, four independent loads in flight per thread.
      constexpr int U = 4;
      constexpr int T = kConsumerThreads;
      const int K4 = static_cast<int>(K / 4);
      if (act.norm_w) {
        for (int r = 0; r < M; ++r) {
          const float4* row = reinterpret_cast<const float4*>(act.x + r * K);
          float ss = 0.0f;
          for (int i0 = ct; i0 < K4; i0 += U * T) {
            float4 t[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
              t[u] = i0 + u * T < K4 ? ld_act(row + i0 + u * T) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < U; ++u) {
              ss = __fmaf_rn(t[u].x, t[u].x, ss);
              ss = __fmaf_rn(t[u].y, t[u].y, ss);
              ss = __fmaf_rn(t[u].z, t[u].z, ss);
              ss = __fmaf_rn(t[u].w, t[u].w, ss);
            }
          }
          ss = consumer_sum(ss, red);
          if (ct == 0) s_inv[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), act.eps)));
        }
        named_bar_sync(1, kConsumerThreads);
      }
      const bool per_row = act.mode == ACT_F32_PER_ROW;
      // Per tensor: one scale over all M rows; per row: one scale per row.
      for (int r0 = 0; r0 < (per_row ? M : 1); ++r0) {
        const int r_lo = per_row ? r0 : 0, r_hi = per_row ? r0 + 1 : M;
        float m = 0.0f;
        for (int r = r_lo; r < r_hi; ++r)
          for (int i0 = ct; i0 < K4; i0 += U * T) {
            float4 t[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
              if (i0 + u * T < K4) t[u] = v.get(r, static_cast<size_t>(i0 + u * T) * 4);
#pragma unroll
            for (int u = 0; u < U; ++u)
              if (i0 + u * T < K4) m = absmax4(m, t[u]);
          }
        const float scale = sym_scale(consumer_max(m, red));
        const float inv = __fdiv_rn(1.0f, scale);
        if (per_row) {
          if (ct == 0) s_scale[r0] = scale;
        } else if (ct < M) {
          s_scale[ct] = scale;
        }
        for (int r = r_lo; r < r_hi; ++r)
          for (int i0 = ct; i0 < K4; i0 += U * T) {
            float4 t[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
              if (i0 + u * T < K4) t[u] = v.get(r, static_cast<size_t>(i0 + u * T) * 4);
#pragma unroll
            for (int u = 0; u < U; ++u)
              if (i0 + u * T < K4) reinterpret_cast<char4*>(s_act)[r * K4 + i0 + u * T] = quant4(t[u], inv);
          }
      }
    } else {
      // Scalar path (unaligned input; no fused producer ops reach here).
      const float* x = act.x;
      for (int r = 0; r < (act.mode == ACT_F32_PER_ROW ? M : 1); ++r) {
        const size_t lo = act.mode == ACT_F32_PER_ROW ? r * K : 0;
        const size_t hi = act.mode == ACT_F32_PER_ROW ? lo + K : total;
        float m = 0.0f;
        for (size_t i = lo + ct; i < hi; i += kConsumerThreads) m = absmax_acc(m, ld_act(x + i));
        const float scale = sym_scale(consumer_max(m, red));
        const float inv = __fdiv_rn(1.0f, scale);
        if (act.mode == ACT_F32_PER_ROW) {
          if (ct == 0) s_scale[r] = scale;
        } else if (ct < M) {
          s_scale[ct] = scale;
        }
        for (size_t i = lo + ct; i < hi; i += kConsumerThreads) s_act[i] = sym_quant(ld_act(x + i), inv);
      }
    }
  } else {
    const int8_t* xq = act.xq;
    if ((reinterpret_cast<uintptr_t>(xq) & 15) == 0 && (total % 16) == 0) {
      for (size_t i = ct; i < total / 16; i += kConsumerThreads)
        reinterpret_cast<uint4*>(s_act)[i] = ld_act(reinterpret_cast<const uint4*>(xq) + i);
    } else {
      for (size_t i = ct; i < total; i += kConsumerThreads) s_act[i] = xq[i];
    }
    if (ct < M) {
      if (act.mode == ACT_I8_HOST_SCALE) s_scale[ct] = act.scale_host;
      else if (act.mode == ACT_I8_DEV_SCALE) s_scale[ct] = ld_act(act.scale_dev);
      else s_scale[ct] = ld_act(act.scale_dev + ct);
    }
  }
  named_bar_sync(1, kConsumerThreads);
}

// ── K2: INT8 per-channel streaming GEMV (K % 16 == 0) ───────────────────────
// Rows are streamed in groups of 8 (one per consumer warp).  When 8 full rows
// would not leave room for three stages, each group is split into nk K-chunks
// of kc bytes: stage (g, c) holds bytes [c*kc, c*kc + kc) of the group's rows,
// copied row by row, and a warp keeps its row's INT32 partial sums in
// registers across the chunks (integer sums: the split is exact).

template <bool CHUNK>
__device__ void stream_producer_i8(const int8_t* W, size_t K, size_t kc, int nk, size_t begin,
                                   size_t end, uint64_t* full, uint64_t* empty, uint8_t* stages_base,
                                   size_t stage_stride, int n_stages, int* status,
                                   uint64_t* act_issued, int pre) {
  const uint64_t policy = l2_policy_evict_first();
  const int groups = static_cast<int>((end - begin + kRowsPerStage - 1) / kRowsPerStage);
  const int iters = groups * nk;
  int issued = 0;
  for (int it = 0; it < iters; ++it) {
    const int s = it % n_stages;
    // Stages after the first `pre` wait until the activation loads are issued.
    if (it == pre && !mbar_wait(act_issued, 0, status)) break;
    if (it >= n_stages) {
      if (!mbar_wait(&empty[s], ((it / n_stages) - 1) & 1, status)) break;
    }
    const int g = it / nk, c = it % nk;
    const size_t r0 = begin + static_cast<size_t>(g) * kRowsPerStage;
    const size_t nrows = std::min<size_t>(kRowsPerStage, end - r0);
    uint8_t* dst = stages_base + s * stage_stride;
    if constexpr (!CHUNK) {
      const uint32_t bytes = static_cast<uint32_t>(nrows * K);
      mbar_arrive_expect_tx(&full[s], bytes);
      bulk_copy_g2s_stream(dst, W + r0 * K, bytes, &full[s], policy);
    } else {
      const size_t k0 = static_cast<size_t>(c) * kc;
      const uint32_t bytes = static_cast<uint32_t>(std::min(kc, K - k0));
      mbar_arrive_expect_tx(&full[s], bytes * static_cast<uint32_t>(nrows));
      for (size_t r = 0; r < nrows; ++r)
        bulk_copy_g2s_stream(dst + r * kc, W + (r0 + r) * K + k0, bytes, &full[s], policy);
    }
    issued = it + 1;
  }
  for (int it = std::max(0, issued - n_stages); it < issued; ++it)
    mbar_wait(&full[it % n_stages], (it / n_stages) & 1, status);
}

// Pair epilogue (EpiArgs): the warps of rows 2i and 2i+1 swap their values
// through shared memory (double-buffered by group parity, one 64-thread named
// barrier per warp pair and group) and combine them.
// pos0: the absolute position of activation row 0; rc, rs: the RoPE cosine
// and sine of this row's pair at that position (rows below qd + kvd), loaded
// by the caller ahead of time.
__device__ __forceinline__ void pair_epilogue(const EpiArgs& epi, int M, size_t N, size_t row,
                                              bool valid, float val, int lane, int cw, int g,
                                              float (*s_pair)[kConsumerWarps][8], float* out,
                                              int pos0, float rc, float rs) {
  if (lane < M) s_pair[g & 1][cw][lane] = val;
  named_bar_sync(2 + (cw >> 1), 64);
  if (!valid || lane >= M) return;
  const float other = s_pair[g & 1][cw ^ 1][lane];
  const int m = lane;
  if (epi.mode == EPI_SWIGLU) {
    // silu(gate) * up (ops/activation/swiglu.rs:39-61, silu.rs:23-26)
    if ((row & 1) == 0) out[m * (N / 2) + row / 2] = swiglu1(val, other);
    return;
  }
  const int r = static_cast<int>(row);
  const int pos = pos0 + m;
  const int qk = epi.qd + epi.kvd;
  float y = val;
  if (r < qk) {
    // ops/rope.rs:121-190: (x0, x1) -> (x0 c - x1 s, x1 c + x0 s), pair j of the head.
    y = (r & 1) == 0 ? __fsub_rn(__fmul_rn(val, rc), __fmul_rn(other, rs))
                     : __fadd_rn(__fmul_rn(val, rc), __fmul_rn(other, rs));
  }
  out[m * N + row] = y;
  if (r >= epi.qd && r < qk) epi.kc[static_cast<size_t>(pos) * epi.kvd + (r - epi.qd)] = y;
  else if (r >= qk) epi.vc[static_cast<size_t>(pos) * epi.kvd + (r - qk)] = y;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// EPI_GATHER tail, consumer threads.  The CTA's output rows were collected in
// shared memory (s_out [M][cap]); they are written to every rank's staging
// with coalesced stores (one remote transfer per 128 bytes instead of one per
// value), fenced, and the CTA counts itself in on every rank's arrival
// counter.  The kernel does not wait: gather_collect_kernel, launched after
// it, waits for the other ranks and copies the result out, so this grid's
// CTAs retire as soon as their rows are done.
// Call state (g_seq, local): [0] arrivals expected after the last call,
// [1] CTA ticket, [2] calls issued (parity = staging half).
template <int M>
__device__ void gather_signal(const EpiArgs& epi, unsigned long long seq, size_t N, size_t begin,
                              size_t end, const float* s_out, int cap) {
  named_bar_sync(1, kConsumerThreads);
  const int ct = threadIdx.x - 32;
  const int rows = static_cast<int>(end - begin);
  const size_t half = (seq & 1) * epi.g_half;
  for (int p = 0; p < epi.g_ranks; ++p)
    for (int m = 0; m < M; ++m) {
      float* dst = epi.g_stage[p] + half + m * epi.g_ntotal + epi.g_rank * N + begin;
      for (int i = ct; i < rows; i += kConsumerThreads) dst[i] = s_out[m * cap + i];
    }
  __threadfence_system();
  named_bar_sync(1, kConsumerThreads);
  if (threadIdx.x == 32) {
    for (int p = 0; p < epi.g_ranks; ++p) atomicAdd_system(epi.g_ctr[p], 1ull);
    __threadfence();
    if (atomicAdd(epi.g_seq + 1, 1ull) == gridDim.x - 1) {
      epi.g_seq[1] = 0;
      epi.g_seq[0] += static_cast<unsigned long long>(epi.g_ranks) * gridDim.x;
      epi.g_seq[2] = seq + 1;
      __threadfence();
    }
  }
}

// CHUNK: rows may be split into nk K-chunks; EPI: 0 none, 1 pair epilogue
// (epi.mode), 2 peer gather.  All compile-time so the plain decode kernel
// carries none of them.
template <int M, int VEC, bool CHUNK, int EPI>
__global__ void __launch_bounds__(kThreads, M <= 2 ? 2 : 1)
    gemv_i8_tma_kernel(const int8_t* __restrict__ W, const float* __restrict__ w_scales, size_t N,
                       size_t K, ActArgs act, float* out, int32_t* __restrict__ acc_out,
                       int n_stages, int nk, int pre, int* status, const float* residual,
                       EpiArgs epi) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float s_pair[2][kConsumerWarps][8];
  if constexpr (!CHUNK) nk = 1;
  const size_t kc = CHUNK ? align_up((K + nk - 1) / nk, 16) : K;
  const StreamLayout L = make_layout(M * K, 0, kRowsPerStage * kc, n_stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + n_stages;
  float* s_scale = reinterpret_cast<float*>(smem + L.scales);
  float* red = s_scale + 8;
  int8_t* s_act = reinterpret_cast<int8_t*>(smem + L.act);
  uint8_t* stage0 = smem + L.stage;

  size_t begin, end;
  // Pair epilogues need both rows of a pair in the same CTA and stage.
  cta_rows(N, EPI == 1 ? 2 : 1, begin, end);
  uint64_t* act_issued = empty + n_stages;
  init_barriers(full, empty, n_stages, act_issued);
  // A gather CTA without rows still takes part in the arrival count.
  if (begin >= end && EPI != 2) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    if (lane == 0)
      stream_producer_i8<CHUNK>(W, K, kc, nk, begin, end, full, empty, stage0, L.stage_bytes, n_stages,
                         status, act_issued, pre);
    return;
  }
  pdl_wait();
  load_act_i8_rowmajor<M, VEC>(act, K, s_act, s_scale, red, act_issued);
  // EPI_GATHER: this CTA's outputs [M][cap], written to all ranks at the end.
  constexpr int kGatherCap = EPI == 2 ? 1024 / M : 1;
  __shared__ float s_gout[EPI == 2 ? 1024 : 1];
  unsigned long long seq = 0;
  if constexpr (EPI == 2) seq = ld_act(epi.g_seq + 2);
  float s_a[M];
#pragma unroll
  for (int m = 0; m < M; ++m) s_a[m] = s_scale[m];

  const int cw = warp - 1;
  const int groups = static_cast<int>((end - begin + kRowsPerStage - 1) / kRowsPerStage);
  // The per-row weight scale, and the epilogue's other global reads (the
  // residual; the RoPE cosine and sine), are loaded one group ahead so their
  // latency overlaps the stage waits and the dot products instead of holding
  // the warp after each group.  (A residual that aliases `out` is read for
  // group g + 1 before group g + 1 writes it.)
  float sw_next = begin + cw < end ? __ldg(w_scales + begin + cw) : 0.0f;
  int pos0 = 0;
  if constexpr (EPI == 1) pos0 = epi.pos_dev ? ld_act(epi.pos_dev) : epi.pos0;
  auto rope_cs = [&](size_t r, float& c, float& sn) {
    c = 0.0f;
    sn = 0.0f;
    if constexpr (EPI == 1) {
      if (epi.mode != EPI_SWIGLU && r < end && static_cast<int>(r) < epi.qd + epi.kvd) {
        const int half = epi.hd / 2, j = (static_cast<int>(r) % epi.hd) >> 1;
        c = __ldg(epi.cos_t + pos0 * half + j);
        sn = __ldg(epi.sin_t + pos0 * half + j);
      }
    }
  };
  auto resid = [&](size_t r) {
    return EPI == 0 && residual && r < end && lane < M ? ld_act(residual + lane * N + r) : 0.0f;
  };
  float rc_next, rs_next;
  rope_cs(begin + cw, rc_next, rs_next);
  float res_next = resid(begin + cw);
  // After a stage wait gives up (status set), the warp still walks the loop
  // without waiting or computing, so every warp reaches the same barriers.
  bool ok = true;
  int it = 0;
  for (int g = 0; g < groups; ++g) {
    const size_t row = begin + static_cast<size_t>(g) * kRowsPerStage + cw;
    const float sw = sw_next;
    if (row + kRowsPerStage < end) sw_next = __ldg(w_scales + row + kRowsPerStage);
    const float rc = rc_next, rs = rs_next, res = res_next;
    rope_cs(row + kRowsPerStage, rc_next, rs_next);
    res_next = resid(row + kRowsPerStage);
    int acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0;
    for (int c = 0; c < nk; ++c, ++it) {
      const int s = it % n_stages;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (it / n_stages) & 1, status));
      if (ok && row < end) {
        const size_t k0 = static_cast<size_t>(c) * kc;
        const int chunks = static_cast<int>(std::min(kc, K - k0) / 16);
        const uint4* wrow = reinterpret_cast<const uint4*>(stage0 + s * L.stage_bytes + cw * kc);
        const int8_t* arow = s_act + k0;
#pragma unroll 4
        for (int q = lane; q < chunks; q += 32) {
          const uint4 w = wrow[q];
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const uint4 a = reinterpret_cast<const uint4*>(arow + m * K)[q];
            acc[m] = dp4a(w.x, a.x, acc[m]);
            acc[m] = dp4a(w.y, a.y, acc[m]);
            acc[m] = dp4a(w.z, a.z, acc[m]);
            acc[m] = dp4a(w.w, a.w, acc[m]);
          }
        }
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&empty[s]);
    }
    const bool valid = ok && row < end;
    float val = 0.0f;
    if (valid) {
#pragma unroll
      for (int m = 0; m < M; ++m) acc[m] = warp_sum_i(acc[m]);
#pragma unroll
      for (int m = 0; m < M; ++m)
        if (lane == m) val = rescale(acc[m], s_a[m], sw);
    }
    if constexpr (EPI == 1) {
      pair_epilogue(epi, M, N, row, valid, val, lane, cw, g, s_pair, out, pos0, rc, rs);
    } else if constexpr (EPI == 2) {
      if (valid && lane < M) s_gout[lane * kGatherCap + (row - begin)] = val;
    } else if (valid && lane < M) {
      // forward_int8.rs:100-121: x + projected (residual may alias out).
      out[lane * N + row] = residual ? __fadd_rn(res, val) : val;
      if (acc_out) {
#pragma unroll
        for (int m = 0; m < M; ++m)
          if (lane == m) acc_out[m * N + row] = acc[m];
      }
    }
  }
  if constexpr (EPI == 2) gather_signal<M>(epi, seq, N, begin, end, s_gout, kGatherCap);
}

// ── generic INT8 GEMV: any K / alignment, pre-quantized activations ─────────

template <int M>
__global__ void __launch_bounds__(256) gemv_i8_generic_kernel(const int8_t* __restrict__ W,
                                                              const float* __restrict__ w_scales,
                                                              size_t N, size_t K, ActArgs act,
                                                              float* __restrict__ out,
                                                              int32_t* __restrict__ acc_out) {
  const int lane = threadIdx.x & 31;
  const size_t warps = static_cast<size_t>(gridDim.x) * (blockDim.x >> 5);
  float s_a[M];
#pragma unroll
  for (int m = 0; m < M; ++m)
    s_a[m] = act.mode == ACT_I8_HOST_SCALE ? act.scale_host
             : act.mode == ACT_I8_DEV_SCALE ? ld_act(act.scale_dev)
                                            : ld_act(act.scale_dev + m);
  for (size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       row < N; row += warps) {
    const int8_t* wr = W + row * K;
    int acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0;
    for (size_t k = lane; k < K; k += 32) {
      const int w = wr[k];
#pragma unroll
      for (int m = 0; m < M; ++m) acc[m] += w * static_cast<int>(act.xq[m * K + k]);
    }
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = warp_sum_i(acc[m]);
    const float sw = w_scales[row];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      if (lane == m) {
        out[m * N + row] = rescale(acc[m], s_a[m], sw);
        if (acc_out) acc_out[m * N + row] = acc[m];
      }
    }
  }
}

// ── K4: Q8_0 streaming GEMV, bit-exact ───────────────────────────────────────
// Activations are quantized per row into shared memory (row-major int8, so
// block b of row m is the 32 bytes at m*K + 32*b).  The 256 consumer threads
// split a stage's (row, block) pairs; a thread keeps the activation bytes of
// its current block in registers (with K = 4096 it never changes block), so
// shared-memory reads are the weight bytes alone.  The block terms
// (f32)dot * s_a * d are computed into registers and the weight stage is
// released at once; the terms then go to a term buffer T[row][m][block], and
// a sum warp adds each (row, m) chain in block order from 0.0, one chain per
// lane (q8_direct.rs:266-285), while the consumers move on to the next stage.
// When a stage has more terms than the consumers' registers hold, they are
// written straight into T after the sum warp has emptied it.

__host__ __device__ constexpr size_t q8_term_stride(size_t nb) { return align_up(nb, 4) + 4; }
constexpr int kQ8Threads = kThreads + 32;  // producer, 8 consumer warps, sum warp
// Terms a consumer thread keeps in registers per activation row (the four of
// K = 4096 at M = 1; a longer unrolled loop costs more than it saves).
__host__ __device__ constexpr int q8_term_regs(int M) { return M >= 4 ? 1 : 4 / M; }
// Shared bytes of the term buffer plus its two mbarriers.
__host__ __device__ constexpr size_t q8_term_bytes(int M, size_t nb) {
  return kConsumerWarps * static_cast<size_t>(M) * q8_term_stride(nb) * sizeof(float) + 16;
}

// Writes the terms tr[i] of units u0 + 256 i (u = row * nb + block) into the
// term buffer T[row][m][block] (row stride M * ts floats).
template <int M, int TR>
__device__ __forceinline__ void q8_store_terms(float* T, uint32_t ts, uint32_t nb, uint32_t u0,
                                               uint32_t rows_here, const float (&tr)[TR][M]) {
  uint32_t r = u0 / nb, b = u0 - r * nb;
  const uint32_t q_step = kConsumerThreads / nb, r_step = kConsumerThreads % nb;
#pragma unroll
  for (int i = 0; i < TR; ++i) {
    if (r >= rows_here) break;  // r never decreases
#pragma unroll
    for (int m = 0; m < M; ++m) T[(r * M + m) * ts + b] = tr[i][m];
    b += r_step;
    r += q_step;
    if (b >= nb) {
      b -= nb;
      ++r;
    }
  }
}

template <int M, int VEC>
__global__ void __launch_bounds__(kQ8Threads, M <= 2 ? 2 : 1)
    gemv_q8_0_tma_kernel(const uint8_t* __restrict__ W, size_t N, size_t K,
                         const float* __restrict__ x, float* __restrict__ out, int n_stages,
                         int pre, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kTR = q8_term_regs(M);
  const size_t nb = K / 32;
  const size_t row_bytes = nb * 34;
  const size_t ts = q8_term_stride(nb);
  const StreamLayout L = make_layout(M * K, q8_term_bytes(M, nb), kRowsPerStage * row_bytes, n_stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + n_stages;
  float* s_scale = reinterpret_cast<float*>(smem + L.scales);
  float* red = s_scale + 8;
  int8_t* s_act = reinterpret_cast<int8_t*>(smem + L.act);
  float* T = reinterpret_cast<float*>(smem + L.extra);  // [8 rows][M][ts]
  uint64_t* tfull = reinterpret_cast<uint64_t*>(smem + L.extra + q8_term_bytes(M, nb) - 16);
  uint64_t* tempty = tfull + 1;
  uint8_t* stage0 = smem + L.stage;

  // Row ranges must start 16-byte aligned: begin * 34 * nb % 16 == 0.
  const size_t g = 8 / (nb % 8 == 0 ? 8 : (nb % 4 == 0 ? 4 : (nb % 2 == 0 ? 2 : 1)));
  size_t begin, end;
  cta_rows(N, g, begin, end);
  uint64_t* act_issued = empty + n_stages;
  if (threadIdx.x == 0) {
    mbar_init(tfull, kConsumerWarps);  // consumers wrote a stage's terms
    mbar_init(tempty, 1);              // the sum warp has added them
  }
  init_barriers(full, empty, n_stages, act_issued);
  if (begin >= end) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int iters = static_cast<int>((end - begin + kRowsPerStage - 1) / kRowsPerStage);
  const uint32_t nb32 = static_cast<uint32_t>(nb), ts32 = static_cast<uint32_t>(ts);
  if (warp == 0) {
    if (lane == 0)
      stream_producer(W, row_bytes, begin, end, full, empty, stage0, L.stage_bytes, n_stages,
                      status, act_issued, pre);
    return;
  }
  pdl_wait();
  if (warp == kConsumerWarps + 1) {
    // Sum warp: chain c = (stage row c / M, activation row c % M).
    for (int it = 0; it < iters; ++it) {
      if (!mbar_wait(tfull, it & 1, status)) return;
      for (int c = lane; c < kRowsPerStage * M; c += 32) {
        const size_t row = begin + static_cast<size_t>(it) * kRowsPerStage + c / M;
        if (row >= end) continue;
        // acc += term in block order (q8_direct.rs:281), starting from 0.0.
        const float* t = T + static_cast<size_t>(c) * ts;
        const float4* t4 = reinterpret_cast<const float4*>(t);
        float acc = 0.0f;
        const uint32_t nb4 = nb32 / 4;
#pragma unroll 8
        for (uint32_t j = 0; j < nb4; ++j) {
          const float4 v = t4[j];
          acc = __fadd_rn(acc, v.x);
          acc = __fadd_rn(acc, v.y);
          acc = __fadd_rn(acc, v.z);
          acc = __fadd_rn(acc, v.w);
        }
        for (uint32_t b = nb4 * 4; b < nb32; ++b) acc = __fadd_rn(acc, t[b]);
        out[static_cast<size_t>(c % M) * N + row] = acc;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
    }
    return;
  }
  // Prologue: per-row quantization (q8_direct.rs:264); one row is one tensor.
  ActArgs act;
  act.x = x;
  act.mode = M == 1 ? ACT_F32_PER_TENSOR : ACT_F32_PER_ROW;
  load_act_i8_rowmajor<M, VEC>(act, K, s_act, s_scale, red, act_issued);
  float s_a[M];
#pragma unroll
  for (int m = 0; m < M; ++m) s_a[m] = s_scale[m];

  // Consumer thread ct takes units u = ct, ct + 256, ... of the stage's
  // (row, block) pairs, u = row * nb + block: for nb = 128 every thread
  // keeps one block (its activation bytes stay in registers) and walks four
  // of the eight rows.
  const uint32_t ct = threadIdx.x - 32;
  const uint32_t kCT = kConsumerThreads;
  const bool buffered = kRowsPerStage * nb32 <= kCT * kTR;
  const uint32_t q_step = kCT / nb32, r_step = kCT % nb32;
  uint32_t xa[M][8];
  uint32_t cur_b = 0xFFFFFFFFu;
  float tr[kTR][M];
  for (int it = 0; it < iters; ++it) {
    const int s = it % n_stages;
    if (!mbar_wait(&full[s], (it / n_stages) & 1, status)) return;
    if (!buffered && it > 0 && !mbar_wait(tempty, (it - 1) & 1, status)) return;
    const size_t r0 = begin + static_cast<size_t>(it) * kRowsPerStage;
    const uint32_t rows_here = static_cast<uint32_t>(std::min<size_t>(kRowsPerStage, end - r0));
    const uint8_t* st = stage0 + s * L.stage_bytes;
    for (uint32_t p0 = 0; p0 < kRowsPerStage * nb32; p0 += kCT * kTR) {
      uint32_t r = (p0 + ct) / nb32, b = (p0 + ct) - r * nb32;
#pragma unroll
      for (int i = 0; i < kTR; ++i) {
        if (r >= rows_here) break;  // r never decreases
        {
          if (b != cur_b) {
            cur_b = b;
#pragma unroll
            for (int m = 0; m < M; ++m) {
              const uint4* a4 = reinterpret_cast<const uint4*>(s_act + m * K + b * 32u);
              const uint4 a0 = a4[0], a1 = a4[1];
              xa[m][0] = a0.x; xa[m][1] = a0.y; xa[m][2] = a0.z; xa[m][3] = a0.w;
              xa[m][4] = a1.x; xa[m][5] = a1.y; xa[m][6] = a1.z; xa[m][7] = a1.w;
            }
          }
          // Block b of row r: 34 bytes at an even address; the words covering
          // it are realigned with one byte permute each.
          const uint8_t* blk = st + r * row_bytes + b * 34u;
          const uint32_t a = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(blk)) & 3u;
          const uint32_t* w = reinterpret_cast<const uint32_t*>(blk - a);
          const uint32_t sel = 0x5432u + (a >> 1) * 0x2222u;
          uint32_t wr[9];
#pragma unroll
          for (int k = 0; k < 9; ++k) wr[k] = w[k];
          const float d = f16_bits_to_f32(__byte_perm(wr[0], 0u, 0x4410u + (a >> 1) * 0x22u));
          uint32_t q[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) q[k] = __byte_perm(wr[k], wr[k + 1], sel);
#pragma unroll
          for (int m = 0; m < M; ++m) {
            int dot = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) dot = dp4a(q[k], xa[m][k], dot);
            tr[i][m] = __fmul_rn(__fmul_rn(small_int_to_float(dot), s_a[m]), d);
          }
        }
        b += r_step;
        r += q_step;
        if (b >= nb32) {
          b -= nb32;
          ++r;
        }
      }
      if (!buffered) q8_store_terms<M, kTR>(T, ts32, nb32, p0 + ct, rows_here, tr);
    }
    // The weights are no longer needed: release the stage before waiting
    // for the sum warp.
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (buffered) {
      if (it > 0 && !mbar_wait(tempty, (it - 1) & 1, status)) return;
      q8_store_terms<M, kTR>(T, ts32, nb32, ct, rows_here, tr);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(tfull);
  }
}

// ── K4, M = 2..8: Q8_0 block dots on the warp-level integer MMA ─────────────
// At M > 1 the block dot products outgrow the CUDA cores: 8 dp4a per
// (weight row, block, activation row).  One mma.sync m16n8k32 (s8 x s8 ->
// s32) computes a block's dots for 8 weight rows (rows 8..15 of the A tile are
// zero) and 8 activation rows at once: A = the 32 quants of row g of the stage
// (groupID g = lane / 4), B = the quantized activation block of row m = g,
// which a dot warp keeps in registers for its whole range of blocks.  Thread
// (g, t = lane % 4) receives the dots of (row g, m = 2t, 2t+1) and writes the
// block terms (f32)dot * s_a * d into a double-buffered term buffer
// [row][block][m]; two sum warps add every (row, m)'s terms in block order
// from 0.0 (q8_direct.rs:266-285), one chain per thread, while the dot warps
// work on the next stage.  The integer dots are exact, so the result is the
// reference's bit for bit.  The dot warps copy the activation rows, quantized
// per row by the quantizer kernel (q8_direct.rs:264), into shared memory while
// the producer streams the first stage.  Rows are copied into stage slots padded by 16 bytes so the 8 rows a
// warp reads fall in different banks.  Preconditions (launcher): nb % 8 == 0,
// nb <= 256.
constexpr int kQ8MmaDotWarps = kConsumerWarps;
constexpr int kQ8MmaSumWarps = 2;
constexpr int kQ8MmaThreads = 32 * (1 + kQ8MmaDotWarps + kQ8MmaSumWarps);
constexpr int kQ8MmaMaxBpw = 32;  // blocks per dot warp (B fragments in registers)
constexpr int kQ8MmaBatch = 8;    // blocks whose shared loads are issued together

__host__ __device__ constexpr size_t q8_mma_row_stride(size_t nb) { return nb * 34 + 16; }
// Floats per stage row in the term buffer: [block][8 m] plus 8 floats of pad.
__host__ __device__ constexpr size_t q8_mma_term_row(size_t nb) { return nb * 8 + 8; }
__host__ __device__ constexpr size_t q8_mma_term_bytes(size_t nb) {
  return 2 * kRowsPerStage * q8_mma_term_row(nb) * sizeof(float);
}

__device__ __forceinline__ void mma_s8_m16n8k32(int d[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                                uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%10, %11, %12, %13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

template <int M>
__global__ void __launch_bounds__(kQ8MmaThreads, 1)
    gemv_q8_0_mma_kernel(const uint8_t* __restrict__ W, size_t N, size_t K,
                         ActArgs act, float* __restrict__ out, int n_stages, int pre,
                         int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  const size_t nb = K / 32;
  const size_t row_bytes = nb * 34;
  const size_t rstride = q8_mma_row_stride(nb);
  const size_t trow = q8_mma_term_row(nb);
  const StreamLayout L = make_layout(q8_mma_term_bytes(nb), 64, kRowsPerStage * rstride, n_stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + n_stages;
  uint64_t* tfull = reinterpret_cast<uint64_t*>(smem + L.extra);  // [2], dot warps arrive
  uint64_t* tempty = tfull + 2;                                    // [2], sum warps arrive
  uint64_t* act_issued = tempty + 2;                               // dot warps' x loads issued
  float* s_scale = reinterpret_cast<float*>(smem + L.scales);
  float* red = s_scale + 8;
  float* T = reinterpret_cast<float*>(smem + L.act);               // [2][8 rows][trow]
  uint8_t* stage0 = smem + L.stage;
  const size_t plane = kRowsPerStage * trow;  // floats per term buffer
  // Until the first stage's terms are written the second term buffer holds
  // the quantized activation rows [M][K].
  int8_t* s_x = reinterpret_cast<int8_t*>(T + plane);

  size_t begin, end;
  cta_rows(N, 1, begin, end);
  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kQ8MmaDotWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], kQ8MmaDotWarps);
      mbar_init(&tempty[b], kQ8MmaSumWarps);
    }
    mbar_init(act_issued, kQ8MmaDotWarps);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  if (begin >= end) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int iters = static_cast<int>((end - begin + kRowsPerStage - 1) / kRowsPerStage);
  if (warp == 0) {
    // Producer: `pre` stages, then the rest once the dot warps have issued
    // their activation loads (so those loads do not queue behind the ring).
    // Each stage row is its own bulk copy into a padded slot.
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      int issued = 0;
      bool ok = true;
      for (int it = 0; it < iters && ok; ++it) {
        const int s = it % n_stages;
        if (it == pre && !mbar_wait(act_issued, 0, status)) break;
        if (it >= n_stages && !mbar_wait(&empty[s], ((it / n_stages) - 1) & 1, status)) {
          ok = false;
          break;
        }
        const size_t r0 = begin + static_cast<size_t>(it) * kRowsPerStage;
        const size_t nrows = std::min<size_t>(kRowsPerStage, end - r0);
        uint8_t* dst = stage0 + s * L.stage_bytes;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nrows * row_bytes));
        for (size_t r = 0; r < nrows; ++r)
          bulk_copy_g2s_stream(dst + r * rstride, W + (r0 + r) * row_bytes,
                               static_cast<uint32_t>(row_bytes), &full[s], policy);
        issued = it + 1;
      }
      for (int it = std::max(0, issued - n_stages); it < issued; ++it)
        mbar_wait(&full[it % n_stages], (it / n_stages) & 1, status);
    }
    return;
  }
  pdl_wait();
  if (warp > kQ8MmaDotWarps) {
    // Sum warps: chain c = (stage row r, activation row m).
    const int c = (warp - 1 - kQ8MmaDotWarps) * 32 + lane;
    const int r = c / M, m = c % M;
    for (int it = 0; it < iters; ++it) {
      const int tb = it & 1;
      if (!mbar_wait(&tfull[tb], (it >> 1) & 1, status)) return;
      const size_t row = begin + static_cast<size_t>(it) * kRowsPerStage + r;
      if (c < kRowsPerStage * M && row < end) {
        const float* t = T + tb * plane + r * trow + m;
        float acc = 0.0f;
#pragma unroll 16
        for (size_t j = 0; j < nb; ++j) acc = __fadd_rn(acc, t[j * 8]);
        out[static_cast<size_t>(m) * N + row] = acc;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[tb]);
    }
    return;
  }

  // Dot warps: warp w owns blocks [w*bpw, (w+1)*bpw); B fragments of its
  // blocks (activation row g, bytes 4t..4t+3 and 16+4t..16+4t+3) stay in
  // registers.
  const int dw = warp - 1;
  const int g = lane >> 2, t = lane & 3;
  const int bpw = static_cast<int>(nb / kQ8MmaDotWarps);
  const int kb0 = dw * bpw;
  // The quantized activation rows into s_x; the prologue ends with a barrier
  // of the dot warps.
  load_act_i8_rowmajor<M, 0>(act, K, s_x, s_scale, red, act_issued);
  uint32_t bf[kQ8MmaMaxBpw][2];
#pragma unroll
  for (int i = 0; i < kQ8MmaMaxBpw; ++i) {
    const bool ok = i < bpw && g < M;
    const uint32_t* p = reinterpret_cast<const uint32_t*>(
        s_x + (ok ? g : 0) * K + static_cast<size_t>(kb0 + (ok ? i : 0)) * 32) + t;
    bf[i][0] = ok ? p[0] : 0u;
    bf[i][1] = ok ? p[4] : 0u;
  }
  const float sa0 = 2 * t < M ? s_scale[2 * t] : 0.0f;
  const float sa1 = 2 * t + 1 < M ? s_scale[2 * t + 1] : 0.0f;
  // The second term buffer is written from stage 1 on: every dot warp has
  // its fragments first.
  named_bar_sync(1, kQ8MmaDotWarps * 32);

  for (int it = 0; it < iters; ++it) {
    const int s = it % n_stages, tb = it & 1;
    if (!mbar_wait(&full[s], (it / n_stages) & 1, status)) return;
    if (it >= 2 && !mbar_wait(&tempty[tb], ((it >> 1) - 1) & 1, status)) return;
    // Row g of the stage (rows past the valid ones hold stale bytes: their
    // terms are written but never summed).
    const uint8_t* rowp = stage0 + s * L.stage_bytes + g * rstride;
    float* Tr = T + tb * plane + g * trow + 2 * t;
    // Batches of kQ8MmaBatch blocks: every shared load of a batch is issued
    // before its term stores (which the compiler cannot move loads across).
#pragma unroll
    for (int i0 = 0; i0 < kQ8MmaMaxBpw; i0 += kQ8MmaBatch) {
      if (i0 >= bpw) break;
      uint32_t a0[kQ8MmaBatch], a2[kQ8MmaBatch], dbits[kQ8MmaBatch];
#pragma unroll
      for (int u = 0; u < kQ8MmaBatch; ++u) {
        // Past the warp's range (bpw not a multiple of the batch) the loads
        // repeat block kb0 and the stores are skipped.
        const int kb = i0 + u < bpw ? kb0 + i0 + u : kb0;
        // Block kb starts at 34*kb, its quants at +2: 2 mod 4 for even kb,
        // word aligned for odd kb (warp-uniform).  Row slots are 4 banks
        // apart, so the 8 rows x 4 threads of a load hit 32 banks.
        const uint8_t* blk = rowp + kb * 34;
        if ((kb & 1) == 0) {
          const uint32_t* w = reinterpret_cast<const uint32_t*>(blk) + t;
          a0[u] = __funnelshift_r(w[0], w[1], 16);
          a2[u] = __funnelshift_r(w[4], w[5], 16);
        } else {
          const uint32_t* w = reinterpret_cast<const uint32_t*>(blk + 2) + t;
          a0[u] = w[0];
          a2[u] = w[4];
        }
        dbits[u] = *reinterpret_cast<const uint16_t*>(blk);
      }
#pragma unroll
      for (int u = 0; u < kQ8MmaBatch; ++u) {
        int dd[4];
        mma_s8_m16n8k32(dd, a0[u], a2[u], bf[i0 + u][0], bf[i0 + u][1]);
        const float d = f16_bits_to_f32(dbits[u]);
        float2 tv;
        tv.x = __fmul_rn(__fmul_rn(small_int_to_float(dd[0]), sa0), d);
        tv.y = __fmul_rn(__fmul_rn(small_int_to_float(dd[1]), sa1), d);
        if (i0 + u < bpw) *reinterpret_cast<float2*>(Tr + (kb0 + i0 + u) * 8) = tv;
      }
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&empty[s]);
      mbar_arrive(&tfull[tb]);
    }
  }
}

// Generic Q8_0: pre-quantized activations in global memory (row-major),
// warp per row, block terms added in order with a lane-serial shuffle chain.
template <int M>
__global__ void __launch_bounds__(256) gemv_q8_0_generic_kernel(const uint8_t* __restrict__ W,
                                                                size_t N, size_t K,
                                                                const int8_t* __restrict__ xq,
                                                                const float* __restrict__ scales,
                                                                float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const size_t nb = K / 32;
  const size_t warps = static_cast<size_t>(gridDim.x) * (blockDim.x >> 5);
  float s_a[M];
#pragma unroll
  for (int m = 0; m < M; ++m) s_a[m] = scales[m];
  for (size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       row < N; row += warps) {
    const uint8_t* rowp = W + row * nb * 34;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.0f;
    for (size_t b0 = 0; b0 < nb; b0 += 32) {
      const size_t b = b0 + lane;
      float t[M];
#pragma unroll
      for (int m = 0; m < M; ++m) t[m] = 0.0f;
      if (b < nb) {
        const uint8_t* blk = rowp + b * 34;
        const float d = f16_bits_to_f32(blk[0] | (blk[1] << 8));
#pragma unroll
        for (int m = 0; m < M; ++m) {
          int dot = 0;
          for (int i = 0; i < 32; ++i)
            dot += static_cast<int>(static_cast<int8_t>(blk[2 + i])) *
                   static_cast<int>(xq[m * K + b * 32 + i]);
          t[m] = __fmul_rn(__fmul_rn(__int2float_rn(dot), s_a[m]), d);
        }
      }
      const int valid = static_cast<int>(std::min<size_t>(32, nb - b0));
      for (int i = 0; i < valid; ++i) {
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = __fadd_rn(acc[m], __shfl_sync(0xffffffffu, t[m], i));
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m)
      if (lane == m) out[m * N + row] = acc[m];
  }
}

// ── K5: Q4_0 streaming GEMV (f32 activations) ───────────────────────────────
// Activations are stored transposed to [m][element 0..31][block] floats.

// Loads the 18-byte Q4_0 block `blk` (at an even address): d (f16 bits) and
// the 16 quant bytes as 4 little-endian words.  The aligned-down word pointer
// is formed by pointer arithmetic on `blk`, so shared loads stay shared.
__device__ __forceinline__ void load_q4_block(const uint8_t* blk, uint32_t& dbits, uint32_t q[4]) {
  const uint32_t a = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(blk)) & 3u;
  const uint32_t* w = reinterpret_cast<const uint32_t*>(blk - a);
  const bool odd = (a & 2) != 0;
  uint32_t r[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) r[i] = w[i];
  dbits = odd ? (r[0] >> 16) : (r[0] & 0xFFFFu);
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = odd ? r[i + 1] : __funnelshift_r(r[i], r[i + 1], 16);
}

// Nibble j (0..3) of the 4 packed in `lo_w`/`hi_w` as an exact float q - 8:
// the byte is placed in the mantissa of 2^23 and 2^23 + 8 subtracted.
__device__ __forceinline__ float nib_minus8(uint32_t v, uint32_t byte_idx) {
  return __int_as_float(static_cast<int>(__byte_perm(v, 0x4B000000u, 0x7540u | byte_idx))) -
         8388616.0f;
}

// Activations (M rows of K floats, consumer threads) into shared memory as
// float4 chunks transposed to [m][chunk 0..7][block], so that lane b reads
// chunk c of block b conflict-free.  Four independent loads in flight per
// thread; each consumer warp arrives on act_issued (when given) once its
// first loads are issued, and the producer holds back later weight stages
// until then.  Ends with a consumer barrier.
template <int M>
__device__ void q4_load_act_f32(const float* __restrict__ x, size_t K, float4* s_x4,
                                uint64_t* act_issued) {
  const size_t nb = K / 32;
  const int lane = threadIdx.x & 31;
  const int ct = threadIdx.x - 32;
  const int K4 = static_cast<int>(K / 4), n4 = M * K4;
  const bool xvec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  constexpr int U = 4;
  const int rounds = (n4 + U * kConsumerThreads - 1) / (U * kConsumerThreads);
  for (int rd = 0; rd < std::max(rounds, 1); ++rd) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = rd * U * kConsumerThreads + u * kConsumerThreads + ct;
      if (idx < n4) {
        if (xvec) {
          v[u] = ld_act(reinterpret_cast<const float4*>(x) + idx);
        } else {
          v[u].x = ld_act(x + 4 * static_cast<size_t>(idx));
          v[u].y = ld_act(x + 4 * static_cast<size_t>(idx) + 1);
          v[u].z = ld_act(x + 4 * static_cast<size_t>(idx) + 2);
          v[u].w = ld_act(x + 4 * static_cast<size_t>(idx) + 3);
        }
      }
    }
    if (rd == 0 && act_issued) {
      __syncwarp();
      if (lane == 0) mbar_arrive(act_issued);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = rd * U * kConsumerThreads + u * kConsumerThreads + ct;
      if (idx < n4) {
        const int r = idx / K4, k = (idx - r * K4) * 4;
        s_x4[(r * 8 + (k % 32) / 4) * nb + k / 32] = v[u];
      }
    }
  }
  named_bar_sync(1, kConsumerThreads);
}

// The f32 Q4_0 product of rows [begin, end) streamed through the stage ring:
// consumer warp w takes row w of each stage, its lanes blocks lane, lane + 32,
// ... (activations from q4_load_act_f32's layout).
template <int M>
__device__ void q4_rows_f32(const float4* s_x4, const uint8_t* stage0, size_t stage_bytes,
                            size_t row_bytes, size_t nb, size_t N, size_t begin, size_t end,
                            uint64_t* full, uint64_t* empty, int n_stages,
                            float* __restrict__ out, int* status) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cw = warp - 1;
  const int iters = static_cast<int>((end - begin + kRowsPerStage - 1) / kRowsPerStage);
  for (int it = 0; it < iters; ++it) {
    const int s = it % n_stages;
    if (!mbar_wait(&full[s], (it / n_stages) & 1, status)) return;
    const size_t row = begin + static_cast<size_t>(it) * kRowsPerStage + cw;
    if (row < end) {
      const uint8_t* rowp = stage0 + s * stage_bytes + cw * row_bytes;
      float acc[M];
#pragma unroll
      for (int m = 0; m < M; ++m) acc[m] = 0.0f;
      const uint32_t nb32 = static_cast<uint32_t>(nb);
      for (uint32_t b = lane; b < nb32; b += 32) {
        uint32_t dbits, q[4];
        load_q4_block(rowp + b * 18u, dbits, q);
        const float d = f16_bits_to_f32(dbits);
        // Per block: sum_k x_k * (q_k - 8), then one multiply by d
        // (dequant_block_into, q4_0.rs:59-68, reassociated).
        float p0[M], p1[M];
#pragma unroll
        for (int m = 0; m < M; ++m) p0[m] = p1[m] = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t w = q[c >> 1];
          const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
          const uint32_t j = (c & 1) * 2;
          const float e0 = nib_minus8(lo, j), e1 = nib_minus8(hi, j);
          const float e2 = nib_minus8(lo, j + 1), e3 = nib_minus8(hi, j + 1);
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const float4 xv = s_x4[(m * 8 + c) * nb32 + b];
            float& p = (c & 1) ? p1[m] : p0[m];
            p = __fmaf_rn(xv.x, e0, p);
            p = __fmaf_rn(xv.y, e1, p);
            p = __fmaf_rn(xv.z, e2, p);
            p = __fmaf_rn(xv.w, e3, p);
          }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = __fmaf_rn(d, p0[m] + p1[m], acc[m]);
      }
#pragma unroll
      for (int m = 0; m < M; ++m) acc[m] = warp_sum_f(acc[m]);
#pragma unroll
      for (int m = 0; m < M; ++m)
        if (lane == m) out[m * N + row] = acc[m];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

template <int M>
__global__ void __launch_bounds__(kThreads, M <= 2 ? 2 : 1)
    gemv_q4_0_tma_kernel(const uint8_t* __restrict__ W, size_t N, size_t K,
                         const float* __restrict__ x, float* __restrict__ out, int n_stages,
                         int pre, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  const size_t nb = K / 32;
  const size_t row_bytes = nb * 18;
  const StreamLayout L = make_layout(M * K * sizeof(float), 0, kRowsPerStage * row_bytes, n_stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + n_stages;
  float4* s_x4 = reinterpret_cast<float4*>(smem + L.act);
  uint8_t* stage0 = smem + L.stage;

  const size_t g = 8 / (nb % 8 == 0 ? 8 : (nb % 4 == 0 ? 4 : (nb % 2 == 0 ? 2 : 1)));
  size_t begin, end;
  cta_rows(N, g, begin, end);
  uint64_t* act_issued = empty + n_stages;
  init_barriers(full, empty, n_stages, act_issued);
  if (begin >= end) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    if (lane == 0)
      stream_producer(W, row_bytes, begin, end, full, empty, stage0, L.stage_bytes, n_stages,
                      status, act_issued, pre);
    return;
  }
  pdl_wait();
  q4_load_act_f32<M>(x, K, s_x4, act_issued);
  q4_rows_f32<M>(s_x4, stage0, L.stage_bytes, row_bytes, nb, N, begin, end, full, empty, n_stages,
                 out, status);
}

// ── K5, M = 1: Q4_0 on exact integer block dots ──────────────────────────────
// The f32 kernel above spends ~4 instructions per weight (nibble -> float,
// FMA, activation reads).  Here the activation row is turned, once per CTA,
// into 21-bit integers per 32-element block: X = rint(x * 2^(19 - e)) with e
// the exponent of the block's largest |x|, so |x - 2^(e-19) X| <= 2^-20 of the
// block maximum, and X is split into three balanced base-128 digits (s8
// planes h, m, l).  A block dot is then exact integer arithmetic: dp4a of the
// unsigned nibbles q against each plane, combined as (h*128 + m)*128 + l,
// minus 8 * sum X (the q - 8 of dequant_block_into, q4_0.rs:59-68).  It is
// scaled by d * 2^(e-19) in f32, and a row's block values are added across
// lanes and warps in a fixed order: the reference's element-by-element f32
// sum (q4_0.rs:94-181) reassociated, within the Q4_0 tolerance.  A row with
// an inf or a NaN takes the f32 kernel's loop instead, so its outputs are
// non-finite where the reference's are.  Consumer thread ct takes units
// u = ct, ct + 256, ... (u = row * nb + block); with nb % 32 == 0 the 32
// lanes of a warp share a row in every unit.  For K = 4096 a thread keeps one
// block, whose digit planes stay in registers.
constexpr int kQ4LimbLoads = 4;   // float4 activation loads per thread in flight
constexpr int kQ4LimbUnroll = 4;  // units per thread in flight (all four of K = 4096)

__host__ __device__ constexpr size_t q4_limb_extra_bytes(size_t K) {
  // digit planes, per-block scale (f32) and digit sum (s32), row partials [2][8][nb / 32]
  return 3 * K + 8 * (K / 32) + 2 * kRowsPerStage * (K / 1024) * sizeof(float);
}

// d = c + sum of (unsigned byte of a) * (signed byte of b).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// X (|X| <= 2^20) as balanced base-128 digits, each in [-64, 64]:
// X = h * 16384 + m * 128 + l.
__device__ __forceinline__ void digits3(int X, int& h, int& m, int& l) {
  l = ((X + 64) & 127) - 64;
  const int x1 = (X - l) >> 7;  // exact: X - l is a multiple of 128
  m = ((x1 + 64) & 127) - 64;
  h = (x1 - m) >> 7;
}

// 2^k for -126 <= k <= 127.
__device__ __forceinline__ float pow2f(int k) { return __int_as_float((k + 127) << 23); }

// v * 2^k, exact while the products stay normal (|v * 2^k| <= 2^20 here).
__device__ __forceinline__ float4 scale_pow2(float4 v, int k) {
  if (k > 127) {
    v = make_float4(v.x * 0x1p127f, v.y * 0x1p127f, v.z * 0x1p127f, v.w * 0x1p127f);
    k -= 127;
  }
  if (k < -126) {
    v = make_float4(v.x * 0x1p-126f, v.y * 0x1p-126f, v.z * 0x1p-126f, v.w * 0x1p-126f);
    k += 126;
  }
  const float f = pow2f(k);
  return make_float4(v.x * f, v.y * f, v.z * f, v.w * f);
}

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | (static_cast<uint32_t>(d) << 24);
}

// Consumer threads: the activation row x[0..K) (16-byte aligned) into the
// digit planes s_l[3][K bytes], the block scales 2^(e-19) and the block digit
// sums.  A plane holds each block's 32 digits in nibble order: the 16 even
// elements, then the 16 odd ones (byte j of a Q4_0 block holds elements 2j
// and 2j + 1), so nibble word k of a block pairs with plane words k and k + 4.  Float4 chunk i holds elements 4i..4i+3 of block i / 8, so the
// 8 lanes of a block reduce with three shuffles.  Returns false (after a
// consumer barrier) when the row holds an inf or a NaN.
__device__ bool q4_limb_prologue(const float* __restrict__ x, size_t K, uint32_t* s_l, float* s_sb,
                                 int* s_S, float* red, uint64_t* act_issued) {
  const int ct = threadIdx.x - 32, lane = threadIdx.x & 31;
  const int K4 = static_cast<int>(K / 4);
  float bad = 0.0f;
  for (int i0 = 0; i0 < K4; i0 += kQ4LimbLoads * kConsumerThreads) {
    float4 v[kQ4LimbLoads];
#pragma unroll
    for (int u = 0; u < kQ4LimbLoads; ++u) {
      const int i = i0 + u * kConsumerThreads + ct;
      v[u] = i < K4 ? ld_act(reinterpret_cast<const float4*>(x) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (i0 == 0 && act_issued) {
      __syncwarp();
      if (lane == 0) mbar_arrive(act_issued);
    }
#pragma unroll
    for (int u = 0; u < kQ4LimbLoads; ++u) {
      const int i = i0 + u * kConsumerThreads + ct;
      const float4 t = v[u];
      if (!(isfinite(t.x) && isfinite(t.y) && isfinite(t.z) && isfinite(t.w))) bad = 1.0f;
      float a = fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w)));
      a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 1));
      a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 2));
      a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 4));
      const int field = static_cast<int>((__float_as_uint(a) >> 23) & 0xFFu);
      const int e = (a > 0.0f && field != 0xFF) ? (field != 0 ? field - 127 : ilogbf(a)) : 0;
      const float4 y = scale_pow2(t, 19 - e);
      const int X0 = __float2int_rn(y.x), X1 = __float2int_rn(y.y);
      const int X2 = __float2int_rn(y.z), X3 = __float2int_rn(y.w);
      int h0, m0, l0, h1, m1, l1, h2, m2, l2, h3, m3, l3;
      digits3(X0, h0, m0, l0);
      digits3(X1, h1, m1, l1);
      digits3(X2, h2, m2, l2);
      digits3(X3, h3, m3, l3);
      int S = X0 + X1 + X2 + X3;
      S += __shfl_xor_sync(0xFFFFFFFFu, S, 1);
      S += __shfl_xor_sync(0xFFFFFFFFu, S, 2);
      S += __shfl_xor_sync(0xFFFFFFFFu, S, 4);
      if (i < K4) {
        // Elements 4c..4c+3 of the block (c = i % 8): the even ones go to
        // bytes 2c, 2c+1 of the block's first 16 bytes, the odd ones to the
        // same bytes of its second 16.
        uint16_t* p = reinterpret_cast<uint16_t*>(s_l) + (i / 8) * 16 + (i % 8);
        const size_t plane = K / 2;  // u16 per digit plane
        p[0] = static_cast<uint16_t>(pack_s8x4(h0, h2, 0, 0));
        p[8] = static_cast<uint16_t>(pack_s8x4(h1, h3, 0, 0));
        p[plane] = static_cast<uint16_t>(pack_s8x4(m0, m2, 0, 0));
        p[plane + 8] = static_cast<uint16_t>(pack_s8x4(m1, m3, 0, 0));
        p[2 * plane] = static_cast<uint16_t>(pack_s8x4(l0, l2, 0, 0));
        p[2 * plane + 8] = static_cast<uint16_t>(pack_s8x4(l1, l3, 0, 0));
        if ((ct & 7) == 0) {
          s_sb[i / 8] = e - 19 >= -126 ? pow2f(e - 19) : scalbnf(1.0f, e - 19);
          s_S[i / 8] = S;
        }
      }
    }
  }
  // The first of consumer_max's barriers also publishes the planes.
  return consumer_max(bad, red) == 0.0f;
}

__global__ void __launch_bounds__(kThreads, 2)
    gemv_q4_0_limb_kernel(const uint8_t* __restrict__ W, size_t N, size_t K,
                          const float* __restrict__ x, float* __restrict__ out, int n_stages,
                          int pre, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  const size_t nb = K / 32;
  const size_t row_bytes = nb * 18;  // a multiple of 16 (nb % 32 == 0)
  const StreamLayout L =
      make_layout(K * sizeof(float), q4_limb_extra_bytes(K), kRowsPerStage * row_bytes, n_stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + n_stages;
  float* red = reinterpret_cast<float*>(smem + L.scales) + 8;
  float4* s_x4 = reinterpret_cast<float4*>(smem + L.act);  // f32 rows (non-finite rows only)
  uint32_t* s_l = reinterpret_cast<uint32_t*>(smem + L.extra);
  float* s_sb = reinterpret_cast<float*>(smem + L.extra + 3 * K);
  int* s_S = reinterpret_cast<int*>(s_sb + nb);
  float* part = reinterpret_cast<float*>(s_S + nb);  // [2][8 rows][nb / 32]
  uint8_t* stage0 = smem + L.stage;

  size_t begin, end;
  cta_rows(N, 1, begin, end);
  uint64_t* act_issued = empty + n_stages;
  init_barriers(full, empty, n_stages, act_issued);
  if (begin >= end) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    if (lane == 0)
      stream_producer(W, row_bytes, begin, end, full, empty, stage0, L.stage_bytes, n_stages,
                      status, act_issued, pre);
    return;
  }
  pdl_wait();
  if (!q4_limb_prologue(x, K, s_l, s_sb, s_S, red, act_issued)) {
    q4_load_act_f32<1>(x, K, s_x4, nullptr);
    q4_rows_f32<1>(s_x4, stage0, L.stage_bytes, row_bytes, nb, N, begin, end, full, empty,
                   n_stages, out, status);
    return;
  }

  const uint32_t ct = threadIdx.x - 32;
  const uint32_t nb32 = static_cast<uint32_t>(nb), K4 = static_cast<uint32_t>(K / 4);
  const uint32_t nbw = nb32 / 32;  // warp units per row
  const uint32_t q_step = kConsumerThreads / nb32, r_step = kConsumerThreads % nb32;
  uint32_t xh[8], xm[8], xl[8];
  float sb = 0.0f;
  int S8 = 0;
  uint32_t cur_b = 0xFFFFFFFFu;
  const int iters = static_cast<int>((end - begin + kRowsPerStage - 1) / kRowsPerStage);
  for (int it = 0; it < iters; ++it) {
    const int s = it % n_stages;
    if (!mbar_wait(&full[s], (it / n_stages) & 1, status)) return;
    const size_t r0 = begin + static_cast<size_t>(it) * kRowsPerStage;
    const uint32_t rows_here = static_cast<uint32_t>(std::min<size_t>(kRowsPerStage, end - r0));
    const uint8_t* st = stage0 + s * L.stage_bytes;
    float* pb = part + (it & 1) * kRowsPerStage * nbw;
    uint32_t r = ct / nb32, b = ct - r * nb32;
    for (uint32_t i0 = 0; i0 < nbw; i0 += kQ4LimbUnroll) {
      // Up to four units, their block values reduced across the warp together.
      float v[kQ4LimbUnroll];
      uint32_t ru[kQ4LimbUnroll], slot[kQ4LimbUnroll];
      if (r_step == 0) {
        // The thread's block never changes (nb divides 256): all the units'
        // loads are issued before any of their arithmetic.
        if (b != cur_b) {
          cur_b = b;
          const uint4* ph = reinterpret_cast<const uint4*>(s_l + 8 * b);
          const uint4* pm = reinterpret_cast<const uint4*>(s_l + K4 + 8 * b);
          const uint4* pl = reinterpret_cast<const uint4*>(s_l + 2 * K4 + 8 * b);
          const uint4 h0 = ph[0], h1 = ph[1], m0 = pm[0], m1 = pm[1], l0 = pl[0], l1 = pl[1];
          xh[0] = h0.x; xh[1] = h0.y; xh[2] = h0.z; xh[3] = h0.w;
          xh[4] = h1.x; xh[5] = h1.y; xh[6] = h1.z; xh[7] = h1.w;
          xm[0] = m0.x; xm[1] = m0.y; xm[2] = m0.z; xm[3] = m0.w;
          xm[4] = m1.x; xm[5] = m1.y; xm[6] = m1.z; xm[7] = m1.w;
          xl[0] = l0.x; xl[1] = l0.y; xl[2] = l0.z; xl[3] = l0.w;
          xl[4] = l1.x; xl[5] = l1.y; xl[6] = l1.z; xl[7] = l1.w;
          sb = s_sb[b];
          S8 = 8 * s_S[b];
        }
        const uint32_t a = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(st + b * 18u)) & 3u;
        const uint32_t sel = 0x5432u + (a >> 1) * 0x2222u;
        uint32_t wr[kQ4LimbUnroll][5];
        bool ok[kQ4LimbUnroll];
#pragma unroll
        for (int u = 0; u < kQ4LimbUnroll; ++u) {
          ru[u] = r + q_step * u;
          slot[u] = b / 32;
          ok[u] = i0 + u < nbw && ru[u] < rows_here;
          const uint32_t* w = reinterpret_cast<const uint32_t*>(
              st + (ok[u] ? ru[u] * row_bytes : 0) + b * 18u - a);
#pragma unroll
          for (int k = 0; k < 5; ++k) wr[u][k] = w[k];
        }
#pragma unroll
        for (int u = 0; u < kQ4LimbUnroll; ++u) {
          const float d = f16_bits_to_f32(__byte_perm(wr[u][0], 0u, 0x4410u + (a >> 1) * 0x22u));
          int dh = 0, dm = 0, dl = 0, eh = 0, em = 0, el = 0;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t q = __byte_perm(wr[u][k], wr[u][k + 1], sel);
            const uint32_t lo = q & 0x0F0F0F0Fu, hi16 = q & 0xF0F0F0F0u;
            dh = dp4a_us(lo, xh[k], dh);
            dm = dp4a_us(lo, xm[k], dm);
            dl = dp4a_us(lo, xl[k], dl);
            eh = dp4a_us(hi16, xh[k + 4], eh);
            em = dp4a_us(hi16, xm[k + 4], em);
            el = dp4a_us(hi16, xl[k + 4], el);
          }
          dh += eh >> 4;
          dm += em >> 4;
          dl += el >> 4;
          const int dot = (dh * 128 + dm) * 128 + dl - S8;
          v[u] = ok[u] ? __fmul_rn(__int2float_rn(dot), __fmul_rn(d, sb)) : 0.0f;
        }
        r += q_step * kQ4LimbUnroll;
      } else {
#pragma unroll
      for (int u = 0; u < kQ4LimbUnroll; ++u) {
        ru[u] = r;
        slot[u] = b / 32;
        v[u] = 0.0f;
        if (i0 + u < nbw && r < rows_here) {  // warp-uniform
          if (b != cur_b) {
            cur_b = b;
            const uint4* ph = reinterpret_cast<const uint4*>(s_l + 8 * b);
            const uint4* pm = reinterpret_cast<const uint4*>(s_l + K4 + 8 * b);
            const uint4* pl = reinterpret_cast<const uint4*>(s_l + 2 * K4 + 8 * b);
            const uint4 h0 = ph[0], h1 = ph[1], m0 = pm[0], m1 = pm[1], l0 = pl[0], l1 = pl[1];
            xh[0] = h0.x; xh[1] = h0.y; xh[2] = h0.z; xh[3] = h0.w;
            xh[4] = h1.x; xh[5] = h1.y; xh[6] = h1.z; xh[7] = h1.w;
            xm[0] = m0.x; xm[1] = m0.y; xm[2] = m0.z; xm[3] = m0.w;
            xm[4] = m1.x; xm[5] = m1.y; xm[6] = m1.z; xm[7] = m1.w;
            xl[0] = l0.x; xl[1] = l0.y; xl[2] = l0.z; xl[3] = l0.w;
            xl[4] = l1.x; xl[5] = l1.y; xl[6] = l1.z; xl[7] = l1.w;
            sb = s_sb[b];
            S8 = 8 * s_S[b];
          }
          // Block b of row r: 18 bytes at an even address (d, then 16 bytes of
          // nibbles: byte j holds elements 2j (low) and 2j + 1 (high),
          // gguf/dequant.rs:471-500).
          const uint8_t* blk = st + r * row_bytes + b * 18u;
          const uint32_t a = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(blk)) & 3u;
          const uint32_t* w = reinterpret_cast<const uint32_t*>(blk - a);
          const uint32_t sel = 0x5432u + (a >> 1) * 0x2222u;
          uint32_t wr[5];
#pragma unroll
          for (int k = 0; k < 5; ++k) wr[k] = w[k];
          const float d = f16_bits_to_f32(__byte_perm(wr[0], 0u, 0x4410u + (a >> 1) * 0x22u));
          // Low nibbles as bytes q, high nibbles left in place as bytes 16 q
          // (their sums are divided by 16 exactly afterwards).
          int dh = 0, dm = 0, dl = 0, eh = 0, em = 0, el = 0;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t q = __byte_perm(wr[k], wr[k + 1], sel);
            const uint32_t lo = q & 0x0F0F0F0Fu, hi16 = q & 0xF0F0F0F0u;
            dh = dp4a_us(lo, xh[k], dh);
            dm = dp4a_us(lo, xm[k], dm);
            dl = dp4a_us(lo, xl[k], dl);
            eh = dp4a_us(hi16, xh[k + 4], eh);
            em = dp4a_us(hi16, xm[k + 4], em);
            el = dp4a_us(hi16, xl[k + 4], el);
          }
          dh += eh >> 4;
          dm += em >> 4;
          dl += el >> 4;
          const int dot = (dh * 128 + dm) * 128 + dl - S8;  // sum (q - 8) X, exact (|dot| < 2^28)
          v[u] = __fmul_rn(__int2float_rn(dot), __fmul_rn(d, sb));
        }
        b += r_step;
        r += q_step;
        if (b >= nb32) {
          b -= nb32;
          ++r;
        }
      }
      }
      // Sum each v[u] over the warp: two halving exchanges leave lane L with a
      // partial of v[(L >> 3) & 3], three more add the lanes of that group.
      const bool up16 = (lane & 16) != 0, up8 = (lane & 8) != 0;
      const float a0 = (up16 ? v[2] : v[0]) + __shfl_xor_sync(0xFFFFFFFFu, up16 ? v[0] : v[2], 16);
      const float a1 = (up16 ? v[3] : v[1]) + __shfl_xor_sync(0xFFFFFFFFu, up16 ? v[1] : v[3], 16);
      float t = (up8 ? a1 : a0) + __shfl_xor_sync(0xFFFFFFFFu, up8 ? a0 : a1, 8);
      t += __shfl_xor_sync(0xFFFFFFFFu, t, 4);
      t += __shfl_xor_sync(0xFFFFFFFFu, t, 2);
      t += __shfl_xor_sync(0xFFFFFFFFu, t, 1);
      if ((lane & 7) == 0) {
        const int u = lane >> 3;  // (up16, up8) -> unit 2 * up16 + up8
        // Register selects (no dynamic indexing into the unit arrays).
        const uint32_t ur = u == 0 ? ru[0] : u == 1 ? ru[1] : u == 2 ? ru[2] : ru[3];
        const uint32_t us = u == 0 ? slot[0] : u == 1 ? slot[1] : u == 2 ? slot[2] : slot[3];
        if (i0 + u < nbw && ur < rows_here) pb[ur * nbw + us] = t;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    // Row r's partials (one per 32 blocks) added in block order.
    named_bar_sync(1, kConsumerThreads);
    if (ct < rows_here) {
      const float* pr = pb + ct * nbw;
      float acc = 0.0f;
      for (uint32_t j = 0; j < nbw; ++j) acc = __fadd_rn(acc, pr[j]);
      out[r0 + ct] = acc;
    }
  }
}

// ── K5, M = 2..8: Q4_0 on the bf16 warp MMA ─────────────────────────────────
// The f32 products of the CUDA-core kernel above are bound by the shared-
// memory reads of the activations (128 bytes per block, weight row and
// activation row).  Here each block's dots for 8 weight rows x 8 activation
// rows are one pair of mma.sync m16n8k16 (bf16 x bf16 -> f32): the weights
// (q - 8, exact in bf16) are the B operand (n = weight row g of the stage, a
// thread's 4 elements of a 16-element k step), and the activations are the A
// operand with rows 0..7 = bf16(x) and rows 8..15 = bf16(x - bf16(x)) of the 8
// activation rows, so one MMA returns both halves of the split and the block
// dot is D[m] + D[m + 8] (16 significant bits of each activation).  A thread's
// k positions are the same in A and B (a0 <-> b0, a2 <-> b1), so any
// assignment of the block's 32 elements to them gives the same dot.  The
// block dot times the block scale d is added to f32 partial sums per (row,
// m); the dot warps' partials are added in warp order by one sum warp.  The
// sum is reassociated (q4_0.rs:94-181 adds element by element): within the
// Q4_0 tolerance.  A pre-kernel writes the split activations in fragment
// order, [m][block][k step j][thread t][a0 a1 a2 a3] holding elements
// 8t + 4j .. 8t + 4j + 3 of the block, rows K*4 + 64 bytes apart
// (the pad puts consecutive rows in opposite bank halves); the producer
// copies them into shared memory once.  Preconditions (launcher): nb % 8 == 0,
// M rows of split activations plus three stages fit.
constexpr int kQ4MmaDotWarps = kConsumerWarps;
constexpr int kQ4MmaThreads = 32 * (1 + kQ4MmaDotWarps + 1);
constexpr int kQ4MmaBatch = 8;

__host__ __device__ constexpr size_t q4_split_row_bytes(size_t K) { return K * 4 + 64; }
__host__ __device__ constexpr size_t q4_mma_row_stride(size_t nb) { return nb * 18 + 16; }
__host__ __device__ constexpr size_t q4_mma_fixed_bytes(int M, size_t K) {
  return static_cast<size_t>(M) * q4_split_row_bytes(K) + 2 * kQ4MmaDotWarps * 64 * sizeof(float);
}

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// x f32 [M, K] -> split bf16 pairs in fragment order (see above); one thread
// per 4 consecutive elements.
__global__ void __launch_bounds__(256) q4_split_act_kernel(const float* __restrict__ x, size_t M,
                                                           size_t K, uint32_t* __restrict__ xs) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t k4 = K / 4;
  if (i >= M * k4) return;
  const size_t m = i / k4, e = (i - m * k4) * 4;
  const float4 v = ld_act(reinterpret_cast<const float4*>(x + m * K + e));
  const float h0 = __bfloat162float(__float2bfloat16_rn(v.x));
  const float h1 = __bfloat162float(__float2bfloat16_rn(v.y));
  const float h2 = __bfloat162float(__float2bfloat16_rn(v.z));
  const float h3 = __bfloat162float(__float2bfloat16_rn(v.w));
  uint4 o;
  o.x = bf16x2_bits(h0, h1);
  o.y = bf16x2_bits(__fsub_rn(v.x, h0), __fsub_rn(v.y, h1));
  o.z = bf16x2_bits(h2, h3);
  o.w = bf16x2_bits(__fsub_rn(v.z, h2), __fsub_rn(v.w, h3));
  // Elements 32*kb + 8*t + 4*j + {0..3} form record (kb, j, t) of row m.
  const size_t kb = e / 32, i4 = (e % 32) / 4, t = i4 >> 1, j = i4 & 1;
  uint8_t* row = reinterpret_cast<uint8_t*>(xs) + m * q4_split_row_bytes(K);
  reinterpret_cast<uint4*>(row)[kb * 8 + j * 4 + t] = o;
}

__device__ __forceinline__ void mma_bf16_m16n8k16(float d[4], const uint4& a, uint32_t b0,
                                                  uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// Four nibble codes (bytes of v, each < 16) as two bf16 pairs q - 8: the code
// goes into the mantissa of bf16(128), then 136 is subtracted (exact).
__device__ __forceinline__ void nib_bf16x2(uint32_t v, uint32_t& p01, uint32_t& p23) {
  const __nv_bfloat162 off = __floats2bfloat162_rn(136.0f, 136.0f);
  uint32_t a = __byte_perm(v, 0x43u, 0x4140), b = __byte_perm(v, 0x43u, 0x4342);
  const __nv_bfloat162 ra = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&a), off);
  const __nv_bfloat162 rb = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&b), off);
  p01 = *reinterpret_cast<const uint32_t*>(&ra);
  p23 = *reinterpret_cast<const uint32_t*>(&rb);
}

template <int M>
__global__ void __launch_bounds__(kQ4MmaThreads, 1)
    gemv_q4_0_mma_kernel(const uint8_t* __restrict__ W, size_t N, size_t K,
                         const uint32_t* __restrict__ xs, float* __restrict__ out, int n_stages,
                         int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  const size_t nb = K / 32;
  const size_t row_bytes = nb * 18;
  const size_t rstride = q4_mma_row_stride(nb);
  const size_t xrow = q4_split_row_bytes(K);
  const StreamLayout L = make_layout(q4_mma_fixed_bytes(M, K), 5 * 8, kRowsPerStage * rstride, n_stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + n_stages;
  uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + L.extra);
  uint64_t* pfull = xfull + 1;   // [2], dot warps arrive
  uint64_t* pempty = pfull + 2;  // [2], the sum warp arrives
  uint8_t* s_x = smem + L.act;   // [M][xrow]
  float* P = reinterpret_cast<float*>(smem + L.act + static_cast<size_t>(M) * xrow);  // [2][8][64]
  uint8_t* stage0 = smem + L.stage;

  size_t begin, end;
  cta_rows(N, 1, begin, end);
  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kQ4MmaDotWarps);
    }
    mbar_init(xfull, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], kQ4MmaDotWarps);
      mbar_init(&pempty[b], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  if (begin >= end) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int iters = static_cast<int>((end - begin + kRowsPerStage - 1) / kRowsPerStage);
  if (warp == 0) {
    // Producer: the whole ring first, then the split activations once the
    // pre-kernel has finished, then the rest of the weights.  Each stage row
    // is its own bulk copy into a padded slot.
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      const int first = std::min(iters, n_stages);
      int issued = 0;
      for (int it = 0; it < iters; ++it) {
        const int s = it % n_stages;
        if (it >= n_stages && !mbar_wait(&empty[s], ((it / n_stages) - 1) & 1, status)) break;
        const size_t r0 = begin + static_cast<size_t>(it) * kRowsPerStage;
        const size_t nrows = std::min<size_t>(kRowsPerStage, end - r0);
        uint8_t* dst = stage0 + s * L.stage_bytes;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nrows * row_bytes));
        for (size_t r = 0; r < nrows; ++r)
          bulk_copy_g2s_stream(dst + r * rstride, W + (r0 + r) * row_bytes,
                               static_cast<uint32_t>(row_bytes), &full[s], policy);
        issued = it + 1;
        if (issued == first) {
          pdl_wait();
          const uint32_t xbytes = static_cast<uint32_t>(M * xrow);
          mbar_arrive_expect_tx(xfull, xbytes);
          bulk_copy_g2s(s_x, xs, xbytes, xfull);
        }
      }
      for (int it = std::max(0, issued - n_stages); it < issued; ++it)
        mbar_wait(&full[it % n_stages], (it / n_stages) & 1, status);
      if (issued >= first) mbar_wait(xfull, 0, status);
    }
    return;
  }
  pdl_wait();
  if (warp > kQ4MmaDotWarps) {
    // Sum warp: output o = m * 8 + n (activation row m, stage row n), the
    // dot warps' partials added in warp order.
    for (int it = 0; it < iters; ++it) {
      const int b = it & 1;
      if (!mbar_wait(&pfull[b], (it >> 1) & 1, status)) return;
      const float* pb = P + b * kQ4MmaDotWarps * 64;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int o = lane + 32 * h, m = o >> 3, n = o & 7;
        float v = pb[o];
#pragma unroll
        for (int w = 1; w < kQ4MmaDotWarps; ++w) v = __fadd_rn(v, pb[w * 64 + o]);
        const size_t row = begin + static_cast<size_t>(it) * kRowsPerStage + n;
        if (m < M && row < end) out[static_cast<size_t>(m) * N + row] = v;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&pempty[b]);
    }
    return;
  }

  // Dot warp w owns blocks [w*bpw, (w+1)*bpw).  Thread (g, t): A rows m = g
  // (hi) and g + 8 (lo); B column n = g (weight row g of the stage); D gives
  // (m = g, n = 2t, 2t + 1).
  const int dw = warp - 1;
  const int g = lane >> 2, t = lane & 3;
  const int bpw = static_cast<int>(nb / kQ4MmaDotWarps);
  const int kb0 = dw * bpw;
  if (!mbar_wait(xfull, 0, status)) return;
  const uint8_t* xa = s_x + static_cast<size_t>(g < M ? g : 0) * xrow;
  const bool arow = g < M;
  for (int it = 0; it < iters; ++it) {
    const int s = it % n_stages, pb = it & 1;
    if (!mbar_wait(&full[s], (it / n_stages) & 1, status)) return;
    const uint8_t* st = stage0 + s * L.stage_bytes;
    const uint8_t* rowg = st + g * rstride;     // B: weight row g
    const uint8_t* row0 = st + 2 * t * rstride;  // block scales of rows 2t, 2t + 1
    float acc0 = 0.0f, acc1 = 0.0f;
    for (int i0 = 0; i0 < bpw; i0 += kQ4MmaBatch) {
      uint32_t wq[kQ4MmaBatch], db[kQ4MmaBatch];
      uint4 a0[kQ4MmaBatch], a1[kQ4MmaBatch];
#pragma unroll
      for (int u = 0; u < kQ4MmaBatch; ++u) {
        // Past the warp's range the loads repeat block kb0; those dots are
        // not added.
        const int kb = i0 + u < bpw ? kb0 + i0 + u : kb0;
        // Block kb starts at 18*kb, its quants at +2: 2 mod 4 for even kb,
        // word aligned for odd kb (warp-uniform).
        const uint8_t* blk = rowg + kb * 18;
        if ((kb & 1) == 0) {
          const uint32_t* w = reinterpret_cast<const uint32_t*>(blk) + t;
          wq[u] = __funnelshift_r(w[0], w[1], 16);
        } else {
          wq[u] = reinterpret_cast<const uint32_t*>(blk + 2)[t];
        }
        const uint8_t* d0 = row0 + kb * 18;
        db[u] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(d0)) |
                (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(d0 + rstride)) << 16);
        const uint4* ar = reinterpret_cast<const uint4*>(xa + static_cast<size_t>(kb) * 128) + t;
        a0[u] = arow ? ar[0] : make_uint4(0u, 0u, 0u, 0u);
        a1[u] = arow ? ar[4] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kQ4MmaBatch; ++u) {
        // Byte i of a Q4_0 block holds elements 2i (low nibble) and 2i + 1
        // (high nibble) (q4_0.rs:59-68): thread t's word holds elements
        // 8t..8t+7, the first four for k step 0 and the rest for k step 1.
        const uint32_t lo = wq[u] & 0x0F0F0F0Fu, hi = (wq[u] >> 4) & 0x0F0F0F0Fu;
        uint32_t b00, b01, b10, b11;
        nib_bf16x2(__byte_perm(lo, hi, 0x5140), b00, b01);  // elements 8t..8t+3
        nib_bf16x2(__byte_perm(lo, hi, 0x7362), b10, b11);  // elements 8t+4..8t+7
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_bf16_m16n8k16(d, a0[u], b00, b01);
        mma_bf16_m16n8k16(d, a1[u], b10, b11);
        if (i0 + u < bpw) {
          acc0 = __fmaf_rn(f16_bits_to_f32(db[u] & 0xFFFFu), __fadd_rn(d[0], d[2]), acc0);
          acc1 = __fmaf_rn(f16_bits_to_f32(db[u] >> 16), __fadd_rn(d[1], d[3]), acc1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (it >= 2 && !mbar_wait(&pempty[pb], ((it >> 1) - 1) & 1, status)) return;
    *reinterpret_cast<float2*>(P + (pb * kQ4MmaDotWarps + dw) * 64 + g * 8 + 2 * t) =
        make_float2(acc0, acc1);
    __syncwarp();
    if (lane == 0) mbar_arrive(&pfull[pb]);
  }
}

template <int M>
__global__ void __launch_bounds__(256) gemv_q4_0_generic_kernel(const uint8_t* __restrict__ W,
                                                                size_t N, size_t K,
                                                                const float* __restrict__ x,
                                                                float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const size_t nb = K / 32;
  const size_t warps = static_cast<size_t>(gridDim.x) * (blockDim.x >> 5);
  for (size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       row < N; row += warps) {
    const uint8_t* rowp = W + row * nb * 18;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.0f;
    for (size_t b = lane; b < nb; b += 32) {
      const uint8_t* blk = rowp + b * 18;
      const float d = f16_bits_to_f32(blk[0] | (blk[1] << 8));
      for (int j = 0; j < 16; ++j) {
        const uint32_t byte = blk[2 + j];
        const float lo = __fmul_rn(d, static_cast<float>(static_cast<int>(byte & 15u) - 8));
        const float hi = __fmul_rn(d, static_cast<float>(static_cast<int>(byte >> 4) - 8));
#pragma unroll
        for (int m = 0; m < M; ++m) {
          acc[m] = __fmaf_rn(ld_act(x + m * K + b * 32 + 2 * j), lo, acc[m]);
          acc[m] = __fmaf_rn(ld_act(x + m * K + b * 32 + 2 * j + 1), hi, acc[m]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = warp_sum_f(acc[m]);
#pragma unroll
    for (int m = 0; m < M; ++m)
      if (lane == m) out[m * N + row] = acc[m];
  }
}

// ── host side: layouts, attributes, dispatch on M ────────────────────────────

int stages_within(size_t fixed_bytes, size_t stage_bytes, size_t budget) {
  for (int s = kMaxStages; s >= 2; --s) {
    const StreamLayout L = make_layout(0, 0, stage_bytes, s);
    if (fixed_bytes + L.total + 256 <= budget) return s;
  }
  return 0;
}

// Stage count and CTAs per SM: two co-resident CTAs of <= 112 KB when at least
// three stages fit (with programmatic dependent launch the next kernel's CTA
// then starts streaming while this one drains), else one CTA of <= 220 KB.
struct StreamConfig {
  int stages = 0;
  int ctas_per_sm = 1;
};

StreamConfig pick_config(size_t fixed_bytes, size_t stage_bytes) {
  StreamConfig c;
  c.stages = std::min(4, stages_within(fixed_bytes, stage_bytes, 112 * 1024));
  if (c.stages >= 3) {
    c.ctas_per_sm = 2;
    return c;
  }
  c.stages = stages_within(fixed_bytes, stage_bytes, kSmemBudget);
  c.ctas_per_sm = 1;
  return c;
}

int pick_stages(size_t fixed_bytes, size_t stage_bytes) {
  return pick_config(fixed_bytes, stage_bytes).stages;
}

size_t fixed_bytes_of(size_t act_bytes, size_t extra_bytes) {
  return align_up(act_bytes, 128) + align_up(extra_bytes, 128) + 256;
}

// Raises a kernel's dynamic shared-memory limit once per (kernel, device,
// size): later launches make no runtime call, so they stay legal inside
// CUDA-graph capture.
template <typename KernelT>
cudaError_t set_smem(KernelT k, size_t bytes, int device) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(reinterpret_cast<const void*>(k), device);
  auto it = done.find(key);
  if (it != done.end() && bytes <= it->second) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(bytes));
  if (e == cudaSuccess) done[key] = bytes;
  return e;
}

int stream_grid(const DeviceInfo& dev, size_t units, int ctas_per_sm) {
  return static_cast<int>(
      std::max<size_t>(1, std::min<size_t>(static_cast<size_t>(dev.sm_count) * ctas_per_sm, units)));
}

// CTAs of `k` that fit on one SM with `smem` dynamic bytes (registers and
// shared memory), cached per (kernel, device, smem).  The persistent grid is
// never sized above it: a second wave would double the kernel's time.
template <typename KernelT>
int resident_ctas(KernelT k, size_t smem, int device, int threads = kThreads) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t>, int> done;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(reinterpret_cast<const void*>(k), device, smem);
  auto it = done.find(key);
  if (it != done.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    n = 1;
  }
  n = std::max(1, n);
  done[key] = n;
  return n;
}

// Launch with the programmatic-stream-serialization attribute when the
// context's MRI_OPT_PDL is on.
template <int Threads = kThreads, typename... KArgs, typename... Args>
cudaError_t launch_stream_kernel(const DeviceInfo& dev, void (*k)(KArgs...), int grid, size_t smem,
                                 cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dev.opt.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_stream_kernel_threads(const DeviceInfo& dev, void (*k)(KArgs...), int grid, int threads,
                                         cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dev.opt.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

#define MRI_DISPATCH_M(M, ...)                           \
  switch (M) {                                           \
    case 1: { constexpr int kM = 1; __VA_ARGS__; } break; \
    case 2: { constexpr int kM = 2; __VA_ARGS__; } break; \
    case 3: { constexpr int kM = 3; __VA_ARGS__; } break; \
    case 4: { constexpr int kM = 4; __VA_ARGS__; } break; \
    case 5: { constexpr int kM = 5; __VA_ARGS__; } break; \
    case 6: { constexpr int kM = 6; __VA_ARGS__; } break; \
    case 7: { constexpr int kM = 7; __VA_ARGS__; } break; \
    case 8: { constexpr int kM = 8; __VA_ARGS__; } break; \
    default: return cudaErrorInvalidValue;               \
  }

}  // namespace

// K-chunk count for the INT8 stream: the smallest nk whose 8 x kc stage
// leaves room for three stages next to the activations.
// Fewest K-chunks that give at least three stages, preferring (up to 16
// chunks) a configuration with two CTAs per SM: their prologues and tails
// overlap each other's streaming.
int i8_chunks(int M, size_t K, StreamConfig* cfg_out) {
  for (int pass = 0; pass < 2; ++pass) {
    for (int nk = 1; nk <= (pass == 0 ? 16 : 64); ++nk) {
      const size_t kc = nk == 1 ? K : align_up((K + nk - 1) / nk, 16);
      if (nk > 1 && kc * (nk - 1) >= K) break;  // chunks would be empty
      const StreamConfig c = pick_config(fixed_bytes_of(M * K, 0), kRowsPerStage * kc);
      if (c.stages >= 3 && (pass == 1 || c.ctas_per_sm >= 2)) {
        if (cfg_out) *cfg_out = c;
        return nk;
      }
    }
  }
  return 0;
}

bool gemv_i8_tma_supported(const DeviceInfo&, int M, size_t K) {
  if (M < 1 || M > 8 || K == 0 || K % 16 != 0) return false;
  return i8_chunks(M, K, nullptr) > 0;
}

// Register-path width for the activation prologue: float4 per consumer
// thread when the input is a per-tensor f32 buffer without SwiGLU and fits
// (4 or 12), else 0 (streamed through the general path).
int reg_vec(int M, size_t K, const ActArgs* act) {
  if (act) {
    if (act->mode != ACT_F32_PER_TENSOR || act->swiglu || K % 4) return 0;
    if ((reinterpret_cast<uintptr_t>(act->x) & 15) ||
        (act->norm_w && (reinterpret_cast<uintptr_t>(act->norm_w) & 15)))
      return 0;
  }
  const size_t per = (static_cast<size_t>(M) * K / 4 + kConsumerThreads - 1) / kConsumerThreads;
  return per <= 4 ? 4 : (per <= 12 ? 12 : 0);
}

#define MRI_DISPATCH_VEC(V, ...)                              \
  switch (V) {                                                \
    case 4: { constexpr int kV = 4; __VA_ARGS__; } break;     \
    case 12: { constexpr int kV = 12; __VA_ARGS__; } break;   \
    default: { constexpr int kV = 0; __VA_ARGS__; } break;    \
  }

// The INT8 stream kernel for (M, VEC, CHUNK, EPI) as `kKernel`.  The pair
// epilogue exists for M = 1 only (the decode step).
#define MRI_DISPATCH_I8_TMA(M, V, CH, EP, ...)                                              \
  if ((EP) == 1) {                                                                          \
    MRI_DISPATCH_VEC(V, {                                                                   \
      if (CH) { auto kKernel = gemv_i8_tma_kernel<1, kV, true, 1>; __VA_ARGS__; }            \
      else { auto kKernel = gemv_i8_tma_kernel<1, kV, false, 1>; __VA_ARGS__; }              \
    });                                                                                     \
  } else if ((EP) == 2) {                                                                   \
    MRI_DISPATCH_M(M, {                                                                     \
      MRI_DISPATCH_VEC(V, {                                                                 \
        if (CH) { auto kKernel = gemv_i8_tma_kernel<kM, kV, true, 2>; __VA_ARGS__; }         \
        else { auto kKernel = gemv_i8_tma_kernel<kM, kV, false, 2>; __VA_ARGS__; }           \
      });                                                                                   \
    });                                                                                     \
  } else {                                                                                  \
    MRI_DISPATCH_M(M, {                                                                     \
      MRI_DISPATCH_VEC(V, {                                                                 \
        if (CH) { auto kKernel = gemv_i8_tma_kernel<kM, kV, true, 0>; __VA_ARGS__; }         \
        else { auto kKernel = gemv_i8_tma_kernel<kM, kV, false, 0>; __VA_ARGS__; }           \
      });                                                                                   \
    });                                                                                     \
  }

// Weight stages a producer issues before the activation loads are in flight:
// one, so that the activation loads of a decode step queue behind one stage
// per CTA instead of the whole ring (swept 0..3 on the 7B decode chain: 488,
// 505, 500, 484 tok/s).
int pre_stages(int stages) { return std::min(1, stages); }

cudaError_t gemv_i8_tma_plan(const DeviceInfo& dev, int M, size_t N, size_t K, GemvPlan* plan,
                             int vec, int epi) {
  if (epi == 1 && M != 1) return cudaErrorInvalidValue;
  StreamConfig cfg;
  const int nk = i8_chunks(M, K, &cfg);
  if (nk == 0 || M < 1 || M > 8) return cudaErrorInvalidValue;
  const size_t kc = nk == 1 ? K : align_up((K + nk - 1) / nk, 16);
  GemvPlan p;
  p.stages = cfg.stages;
  p.k_chunks = nk;
  p.vec = vec < 0 ? reg_vec(M, K, nullptr) : vec;
  p.smem = make_layout(M * K, 0, kRowsPerStage * kc, p.stages).total;
  p.epi = epi;
  MRI_DISPATCH_I8_TMA(M, p.vec, nk > 1, epi, {
    cudaError_t e = set_smem(kKernel, p.smem, dev.device);
    if (e != cudaSuccess) return e;
    p.resident = resident_ctas(kKernel, p.smem, dev.device);
  });
  p.ctas_per_sm = std::min(cfg.ctas_per_sm, p.resident);
  p.grid = stream_grid(dev, N, p.ctas_per_sm);
  *plan = p;
  return cudaSuccess;
}

cudaError_t launch_gemv_i8_tma(const DeviceInfo& dev, cudaStream_t st, int M, const int8_t* W,
                               const float* w_scales, size_t N, size_t K, const ActArgs& act,
                               float* out, int32_t* acc_out, int* status, LaunchStats* ls,
                               const float* residual, const EpiArgs* epi) {
  EpiArgs e_args;
  int kind = 0;
  if (epi) {
    kind = epi->mode == EPI_GATHER ? 2 : 1;
    if ((kind == 1 && N % 2) || residual || acc_out) return cudaErrorInvalidValue;
    if (kind == 2 && (epi->g_ranks < 1 || epi->g_ranks > EpiArgs::kMaxRanks)) return cudaErrorInvalidValue;
    e_args = *epi;
  }
  GemvPlan p;
  if (cudaError_t e = gemv_i8_tma_plan(dev, M, N, K, &p, reg_vec(M, K, &act), kind)) return e;
  // A gather CTA keeps its output rows in a 1024-float shared buffer.
  if (kind == 2 && ((N + p.grid - 1) / p.grid) * M > 1024) return cudaErrorInvalidValue;
  const int pre = act.pre_stages >= 0 ? std::min(act.pre_stages, p.stages) : pre_stages(p.stages);
  MRI_DISPATCH_I8_TMA(M, p.vec, p.k_chunks > 1, p.epi, {
    // The gather CTAs wait for one another, so all must be resident at once:
    // the grid never exceeds the CTAs that fit (resident_ctas), and a
    // dependent launch can only start once every CTA of this grid has
    // started.  A cooperative launch would also serialise it against the
    // previous kernel, which costs more than the wait saves.
    cudaError_t e = launch_stream_kernel(dev, kKernel, p.grid, p.smem, st, W, w_scales, N, K, act, out,
                                         acc_out, p.stages, p.k_chunks, pre, status, residual, e_args);
    if (e != cudaSuccess) return e;
  });
  if (ls) ls->launches++;
  return cudaGetLastError();
}

// Second half of the peer gather: wait (bounded) until every rank's CTAs of the
// preceding gather GEMV have arrived on the local counter, then copy the
// assembled [M][n_total] result from the staging half of that call to out.
__global__ void __launch_bounds__(256) gather_collect_kernel(const unsigned long long* ctr,
                                                             const unsigned long long* call,
                                                             const float* stage, size_t half,
                                                             size_t total, float* out, int* status) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ int s_ok;
  const unsigned long long target = ld_act(call);
  const unsigned long long issued = ld_act(call + 2);
  if (threadIdx.x == 0) {
    int ok = 1;
    const long long t0 = clock64();
    while (ld_acquire_sys_u64(ctr) < target) {
      if (clock64() - t0 > kWaitBudgetClocks) {
        *reinterpret_cast<volatile int*>(status) = MRI_ERR_TIMEOUT;
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const float* src = stage + ((issued - 1) & 1) * half;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total; i += stride)
    out[i] = ld_act(src + i);
}

cudaError_t launch_gather_collect(const DeviceInfo& dev, cudaStream_t st, const EpiArgs& e, int M,
                                  int* status, LaunchStats* ls) {
  const size_t total = static_cast<size_t>(M) * e.g_ntotal;
  const int grid = static_cast<int>(std::max<size_t>(1, std::min<size_t>(dev.sm_count, (total + 1023) / 1024)));
  cudaError_t err = launch_stream_kernel_threads(dev, gather_collect_kernel, grid, 256, st,
                                                 static_cast<const unsigned long long*>(e.g_ctr[e.g_rank]),
                                                 static_cast<const unsigned long long*>(e.g_seq),
                                                 static_cast<const float*>(e.g_stage[e.g_rank]), e.g_half, total,
                                                 e.g_out, status);
  if (ls) ls->launches++;
  return err;
}

cudaError_t launch_gemv_i8_generic(const DeviceInfo& dev, cudaStream_t st, int M, const int8_t* W,
                                   const float* w_scales, size_t N, size_t K, const ActArgs& act,
                                   float* out, int32_t* acc_out, LaunchStats* ls) {
  const int grid = static_cast<int>(std::max<size_t>(1, std::min<size_t>((N + 7) / 8, dev.sm_count * 8)));
  MRI_DISPATCH_M(M, {
    gemv_i8_generic_kernel<kM><<<grid, 256, 0, st>>>(W, w_scales, N, K, act, out, acc_out);
  });
  if (ls) ls->launches++;
  return cudaGetLastError();
}

bool gemv_q8_0_tma_supported(const DeviceInfo&, int M, size_t K) {
  if (M < 1 || M > 8 || K == 0 || K % 32 != 0) return false;
  const size_t nb = K / 32;
  return pick_stages(fixed_bytes_of(M * K, q8_term_bytes(M, nb)),
                     kRowsPerStage * nb * 34) >= 3;
}

// The MMA Q8_0 kernel covers M = 2..8 when nb % 8 == 0 (16-byte aligned
// rows, an equal block range per dot warp), nb <= 8 * kQ8MmaMaxBpw and three
// stages fit.
bool q8_0_mma_supported(const DeviceInfo& dev, int M, size_t K) {
  if (!dev.opt.q8_mma || M < 2 || M > 8 || K == 0 || K % 32 != 0) return false;
  const size_t nb = K / 32;
  if (nb % kQ8MmaDotWarps != 0 || nb > static_cast<size_t>(kQ8MmaDotWarps * kQ8MmaMaxBpw)) return false;
  return stages_within(fixed_bytes_of(q8_mma_term_bytes(nb), 64), kRowsPerStage * q8_mma_row_stride(nb),
                       kSmemBudget) >= 3;
}

cudaError_t launch_gemv_q8_0_mma(const DeviceInfo& dev, cudaStream_t st, int M, const uint8_t* W,
                                 size_t N, size_t K, const ActArgs& act, float* out, int* status,
                                 LaunchStats* ls) {
  if (!q8_0_mma_supported(dev, M, K) || (reinterpret_cast<uintptr_t>(W) & 15) != 0 ||
      act.mode != ACT_I8_DEV_ROW_SCALE)
    return cudaErrorInvalidValue;
  const size_t nb = K / 32;
  const size_t stage_bytes = kRowsPerStage * q8_mma_row_stride(nb);
  const int stages = std::min(kMaxStages, stages_within(fixed_bytes_of(q8_mma_term_bytes(nb), 64),
                                                         stage_bytes, kSmemBudget));
  const size_t smem = make_layout(q8_mma_term_bytes(nb), 64, stage_bytes, stages).total;
  void (*kern)(const uint8_t*, size_t, size_t, ActArgs, float*, int, int, int*) = nullptr;
  switch (M) {
    case 2: kern = gemv_q8_0_mma_kernel<2>; break;
    case 3: kern = gemv_q8_0_mma_kernel<3>; break;
    case 4: kern = gemv_q8_0_mma_kernel<4>; break;
    case 5: kern = gemv_q8_0_mma_kernel<5>; break;
    case 6: kern = gemv_q8_0_mma_kernel<6>; break;
    case 7: kern = gemv_q8_0_mma_kernel<7>; break;
    case 8: kern = gemv_q8_0_mma_kernel<8>; break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = set_smem(kern, smem, dev.device);
  if (e != cudaSuccess) return e;
  // Weight stages issued before the activation loads: the whole ring at 8
  // rows (measured per [11008, 4096] call: 20.0 -> 19.4 us), one below (M = 4:
  // 18.3 us with the whole ring, 18.0 with one; M = 2: 18.2 and 17.7).
  const int pre = M >= 8 ? stages : pre_stages(stages);
  e = launch_stream_kernel<kQ8MmaThreads>(dev, kern, stream_grid(dev, N, 1), smem, st, W, N, K, act,
                                          out, stages, pre, status);
  if (e != cudaSuccess) return e;
  if (ls) ls->launches++;
  return cudaGetLastError();
}

cudaError_t launch_gemv_q8_0_tma(const DeviceInfo& dev, cudaStream_t st, int M, const uint8_t* W,
                                 size_t N, size_t K, const float* x, float* out, int* status,
                                 LaunchStats* ls) {
  const size_t nb = K / 32;
  const size_t extra = q8_term_bytes(M, nb);
  const StreamConfig cfg = pick_config(fixed_bytes_of(M * K, extra), kRowsPerStage * nb * 34);
  const int stages = cfg.stages;
  if (stages < 2) return cudaErrorInvalidValue;
  const size_t smem = make_layout(M * K, extra, kRowsPerStage * nb * 34, stages).total;
  // M = 1: per-row is per-tensor, so the register prologue applies.
  ActArgs probe;
  probe.x = x;
  const int vec = M == 1 ? reg_vec(1, K, &probe) : 0;
  const int pre = pre_stages(stages);
  MRI_DISPATCH_M(M, {
    MRI_DISPATCH_VEC(M == 1 ? vec : 0, {
      auto kern = gemv_q8_0_tma_kernel<kM, (kM == 1 ? kV : 0)>;
      cudaError_t e = set_smem(kern, smem, dev.device);
      if (e != cudaSuccess) return e;
      const int grid = stream_grid(
          dev, N, std::min(cfg.ctas_per_sm, resident_ctas(kern, smem, dev.device, kQ8Threads)));
      e = launch_stream_kernel<kQ8Threads>(dev, kern, grid, smem, st, W, N, K, x, out, stages, pre,
                                           status);
      if (e != cudaSuccess) return e;
    });
  });
  if (ls) ls->launches++;
  return cudaGetLastError();
}

cudaError_t launch_gemv_q8_0_generic(const DeviceInfo& dev, cudaStream_t st, int M,
                                     const uint8_t* W, size_t N, size_t K, const int8_t* xq,
                                     const float* scales, float* out, LaunchStats* ls) {
  const int grid = static_cast<int>(std::max<size_t>(1, std::min<size_t>((N + 7) / 8, dev.sm_count * 8)));
  MRI_DISPATCH_M(M, {
    gemv_q8_0_generic_kernel<kM><<<grid, 256, 0, st>>>(W, N, K, xq, scales, out);
  });
  if (ls) ls->launches++;
  return cudaGetLastError();
}

bool gemv_q4_0_tma_supported(const DeviceInfo&, int M, size_t K) {
  if (M < 1 || M > 8 || K == 0 || K % 32 != 0) return false;
  return pick_stages(fixed_bytes_of(M * K * 4, 0), kRowsPerStage * (K / 32) * 18) >= 3;
}

cudaError_t launch_gemv_q4_0_tma(const DeviceInfo& dev, cudaStream_t st, int M, const uint8_t* W,
                                 size_t N, size_t K, const float* x, float* out, int* status,
                                 LaunchStats* ls) {
  const size_t stage_bytes = kRowsPerStage * (K / 32) * 18;
  const StreamConfig cfg = pick_config(fixed_bytes_of(M * K * 4, 0), stage_bytes);
  const int stages = cfg.stages;
  if (stages < 2) return cudaErrorInvalidValue;
  const size_t smem = make_layout(M * K * 4, 0, stage_bytes, stages).total;
  MRI_DISPATCH_M(M, {
    cudaError_t e = set_smem(gemv_q4_0_tma_kernel<kM>, smem, dev.device);
    if (e != cudaSuccess) return e;
    const int grid = stream_grid(
        dev, N, std::min(cfg.ctas_per_sm, resident_ctas(gemv_q4_0_tma_kernel<kM>, smem, dev.device)));
    e = launch_stream_kernel(dev, gemv_q4_0_tma_kernel<kM>, grid, smem, st, W, N, K, x, out, stages,
                             pre_stages(stages), status);
    if (e != cudaSuccess) return e;
  });
  if (ls) ls->launches++;
  return cudaGetLastError();
}

static StreamConfig q4_0_limb_config(size_t K) {
  return pick_config(fixed_bytes_of(K * sizeof(float), q4_limb_extra_bytes(K)),
                     kRowsPerStage * (K / 32) * 18);
}

bool gemv_q4_0_limb_supported(const DeviceInfo& dev, size_t K, const float* x) {
  if (!dev.opt.q4_limb || K == 0 || K % 1024 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return false;
  return q4_0_limb_config(K).stages >= 3;
}

cudaError_t launch_gemv_q4_0_limb(const DeviceInfo& dev, cudaStream_t st, const uint8_t* W, size_t N,
                                  size_t K, const float* x, float* out, int* status, LaunchStats* ls) {
  if (!gemv_q4_0_limb_supported(dev, K, x)) return cudaErrorInvalidValue;
  const StreamConfig cfg = q4_0_limb_config(K);
  const size_t stage_bytes = kRowsPerStage * (K / 32) * 18;
  const size_t smem =
      make_layout(K * sizeof(float), q4_limb_extra_bytes(K), stage_bytes, cfg.stages).total;
  cudaError_t e = set_smem(gemv_q4_0_limb_kernel, smem, dev.device);
  if (e != cudaSuccess) return e;
  const int grid = stream_grid(
      dev, N, std::min(cfg.ctas_per_sm, resident_ctas(gemv_q4_0_limb_kernel, smem, dev.device)));
  e = launch_stream_kernel(dev, gemv_q4_0_limb_kernel, grid, smem, st, W, N, K, x, out, cfg.stages,
                           pre_stages(cfg.stages), status);
  if (e != cudaSuccess) return e;
  if (ls) ls->launches++;
  return cudaGetLastError();
}

// The bf16-MMA Q4_0 kernel covers M = 2..8 when nb % 8 == 0 (16-byte aligned
// rows, an equal block range per dot warp) and the split activations plus
// three stages fit.
int q4_0_mma_stages(int M, size_t K) {
  const size_t nb = K / 32;
  return std::min(kMaxStages, stages_within(fixed_bytes_of(q4_mma_fixed_bytes(M, K), 5 * 8),
                                            kRowsPerStage * q4_mma_row_stride(nb), kSmemBudget));
}

bool q4_0_mma_supported(const DeviceInfo& dev, int M, size_t K) {
  if (!dev.opt.q4_mma || M < 2 || M > 8 || K == 0 || K % 32 != 0) return false;
  if ((K / 32) % kQ4MmaDotWarps != 0) return false;
  return q4_0_mma_stages(M, K) >= 3;
}

size_t q4_0_split_bytes(size_t m, size_t K) { return m * q4_split_row_bytes(K); }

cudaError_t launch_q4_0_split(const DeviceInfo& dev, cudaStream_t st, const float* x, size_t m, size_t K,
                              uint32_t* xs, LaunchStats* ls) {
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (reinterpret_cast<uintptr_t>(xs) & 15) != 0 ||
      K % 4 != 0)
    return cudaErrorInvalidValue;
  const size_t n4 = m * (K / 4);
  if (n4 == 0) return cudaSuccess;
  const int grid = static_cast<int>((n4 + 255) / 256);
  cudaError_t e = launch_stream_kernel_threads(dev, q4_split_act_kernel, grid, 256, st, x, m, K, xs);
  if (ls) ls->launches++;
  return e;
}

cudaError_t launch_gemv_q4_0_mma(const DeviceInfo& dev, cudaStream_t st, int M, const uint8_t* W,
                                 size_t N, size_t K, const uint32_t* xs, float* out, int* status,
                                 LaunchStats* ls) {
  if (!q4_0_mma_supported(dev, M, K) || (reinterpret_cast<uintptr_t>(xs) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(W) & 15) != 0)
    return cudaErrorInvalidValue;
  const size_t nb = K / 32;
  const int stages = q4_0_mma_stages(M, K);
  const size_t smem =
      make_layout(q4_mma_fixed_bytes(M, K), 5 * 8, kRowsPerStage * q4_mma_row_stride(nb), stages).total;
  void (*kern)(const uint8_t*, size_t, size_t, const uint32_t*, float*, int, int*) = nullptr;
  switch (M) {
    case 2: kern = gemv_q4_0_mma_kernel<2>; break;
    case 3: kern = gemv_q4_0_mma_kernel<3>; break;
    case 4: kern = gemv_q4_0_mma_kernel<4>; break;
    case 5: kern = gemv_q4_0_mma_kernel<5>; break;
    case 6: kern = gemv_q4_0_mma_kernel<6>; break;
    case 7: kern = gemv_q4_0_mma_kernel<7>; break;
    case 8: kern = gemv_q4_0_mma_kernel<8>; break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = set_smem(kern, smem, dev.device);
  if (e != cudaSuccess) return e;
  e = launch_stream_kernel<kQ4MmaThreads>(dev, kern, stream_grid(dev, N, 1), smem, st, W, N, K, xs, out,
                                          stages, status);
  if (e != cudaSuccess) return e;
  if (ls) ls->launches++;
  return cudaGetLastError();
}

cudaError_t launch_gemv_q4_0_generic(const DeviceInfo& dev, cudaStream_t st, int M,
                                     const uint8_t* W, size_t N, size_t K, const float* x,
                                     float* out, LaunchStats* ls) {
  const int grid = static_cast<int>(std::max<size_t>(1, std::min<size_t>((N + 7) / 8, dev.sm_count * 8)));
  MRI_DISPATCH_M(M, {
    gemv_q4_0_generic_kernel<kM><<<grid, 256, 0, st>>>(W, N, K, x, out);
  });
  if (ls) ls->launches++;
  return cudaGetLastError();
}

}  // namespace mri
