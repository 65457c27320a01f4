// llama.cu — device-resident LlamaModelInt8 (model/llama/forward_int8.rs:
// 148-547) around the quantized projections: the caller of the hot path for
// the full-model config (32 layers, 512-token prefill, greedy decode).
//
// Everything stays on the GPU: embeddings, norms, RoPE tables, the flat f32
// KV cache ([layer][max_seq][kv_dim], cache/kv_cache.rs:44-175), activations.
// Each projection is the library's INT8 product with the reference's
// per-tensor activation quantization (proj_int8, forward_int8.rs:72-96):
// small token counts take the fused streaming GEMV, prefill the tcgen05 GEMM.
// Q, K and V (and gate and up) weights are stored as one concatenated
// QuantizedMatrix; since each projection quantizes the same input with the
// same per-tensor scale, every output element is bit-identical to separate
// calls.  RMSNorm and SwiGLU run fused in front of the projection that
// consumes them (inside the activation-quantization prologue) and the
// residual add behind it (in the product's epilogue); RoPE, attention and the
// greedy argmax are plain CUDA.  The glue is f32 and tolerance-checked, not
// bit-exact (its exp/sum order differs from the reference's).
//
// A decode step reads the token and position from device memory, so one
// captured CUDA graph replays every step of greedy generation.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <utility>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <string>
#include <vector>

#include <cooperative_groups.h>

#include "common.cuh"
#include "internal.h"
#include "mri_gpu.h"

namespace cg = cooperative_groups;

namespace {

constexpr int kPrefillQ = 16;    // queries per block in prefill attention
constexpr int kPrefillKT = 64;   // keys per shared-memory tile in prefill attention
constexpr int kMaxHeadDim = 128;

// ── glue kernels ─────────────────────────────────────────────────────────────
// The decode-step kernels are launched with programmatic dependent launch:
// each lets its successor be scheduled early (pdl_trigger) and touches memory
// only after griddepcontrol.wait, which returns once the predecessor grid has
// completed and its writes are visible.

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// forward_int8.rs:125-140 (row copy); token ids are validated on the host for
// host-supplied tokens and are < vocab by construction for argmax outputs.
__global__ void embed_kernel(const uint32_t* __restrict__ tokens, const float* __restrict__ embd,
                             int d, float* __restrict__ x) {
  pdl_trigger();
  pdl_wait();
  const uint32_t tok = mri::ld_act(tokens + blockIdx.x);
  const float* src = embd + static_cast<size_t>(tok) * d;
  float* dst = x + static_cast<size_t>(blockIdx.x) * d;
  if ((d & 3) == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
    // The row in 16-byte pieces, up to 8 loads in flight per thread before
    // any store (one HBM round trip for a 4096-wide row).
    constexpr int U = 8;
    const int d4 = d / 4;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* o4 = reinterpret_cast<float4*>(dst);
    for (int i0 = 0; i0 < d4; i0 += U * static_cast<int>(blockDim.x)) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * static_cast<int>(blockDim.x) + static_cast<int>(threadIdx.x);
        if (i < d4) v[u] = s4[i];
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * static_cast<int>(blockDim.x) + static_cast<int>(threadIdx.x);
        if (i < d4) o4[i] = v[u];
      }
    }
    return;
  }
  for (int i = threadIdx.x; i < d; i += blockDim.x) dst[i] = src[i];
}

// ops/rope.rs:121-190 on q and k of the fused qkv rows, then the cache write
// of attention/cached.rs:90-93 / :161-163 (k rotated, v as is).  Block
// (i, h): head h of token row i at absolute position base + i, where base is
// *pos_dev if given, else pos0; heads [0, H) are queries, [H, H+Hkv) keys
// (whose blocks also copy the matching value head into the cache).
// Prefill form: block i takes token row i whole (all query and key heads and
// the value copy), four elements (two rotation pairs) per thread step, the
// same arithmetic per element.  hd % 4 == 0, ld % 4 == 0, 16-byte aligned
// rows and caches.
__global__ void __launch_bounds__(256) rope_kv_rows_kernel(float* __restrict__ qkv, int ld, int n_heads,
                                                           int n_kv, int hd,
                                                           const float* __restrict__ cos_t,
                                                           const float* __restrict__ sin_t, int pos0,
                                                           float* __restrict__ kc, float* __restrict__ vc) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  const int pos = pos0 + i;
  const int half = hd / 2;
  float* row = qkv + static_cast<size_t>(i) * ld;
  const int kvd = n_kv * hd, qd = n_heads * hd;
  const float* cr = cos_t + static_cast<size_t>(pos) * half;
  const float* sr = sin_t + static_cast<size_t>(pos) * half;
  float* krow = kc + static_cast<size_t>(pos) * kvd;
  float* vrow = vc + static_cast<size_t>(pos) * kvd;
  // q and k: elements e..e+3 of the (qd + kvd)-wide rotated part.
  for (int e = threadIdx.x * 4; e < qd + kvd; e += blockDim.x * 4) {
    const int j = (e % hd) / 2;  // first of the two pairs
    float4 v = mri::ld_act(reinterpret_cast<const float4*>(row + e));
    const float2 c = *reinterpret_cast<const float2*>(cr + j);
    const float2 sn = *reinterpret_cast<const float2*>(sr + j);
    float4 y;
    y.x = __fsub_rn(__fmul_rn(v.x, c.x), __fmul_rn(v.y, sn.x));
    y.y = __fadd_rn(__fmul_rn(v.y, c.x), __fmul_rn(v.x, sn.x));
    y.z = __fsub_rn(__fmul_rn(v.z, c.y), __fmul_rn(v.w, sn.y));
    y.w = __fadd_rn(__fmul_rn(v.w, c.y), __fmul_rn(v.z, sn.y));
    *reinterpret_cast<float4*>(row + e) = y;
    if (e >= qd) *reinterpret_cast<float4*>(krow + (e - qd)) = y;
  }
  for (int e = threadIdx.x * 4; e < kvd; e += blockDim.x * 4)
    *reinterpret_cast<float4*>(vrow + e) = mri::ld_act(reinterpret_cast<const float4*>(row + qd + kvd + e));
}

__global__ void rope_kv_kernel(float* __restrict__ qkv, int ld, int n_heads, int n_kv, int hd,
                               const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                               int pos0, const int* __restrict__ pos_dev, float* __restrict__ kc,
                               float* __restrict__ vc) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x, h = blockIdx.y;
  const int pos = (pos_dev ? mri::ld_act(pos_dev) : pos0) + i;
  const int half = hd / 2;
  float* row = qkv + static_cast<size_t>(i) * ld;
  const int kvd = n_kv * hd, qd = n_heads * hd;
  float* base = h < n_heads ? row + h * hd : row + qd + (h - n_heads) * hd;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float c = cos_t[pos * half + j], sn = sin_t[pos * half + j];
    const float x0 = mri::ld_act(base + 2 * j), x1 = mri::ld_act(base + 2 * j + 1);
    const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
    const float y1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn));
    base[2 * j] = y0;
    base[2 * j + 1] = y1;
    if (h >= n_heads) {
      const int kh = h - n_heads;
      float* krow = kc + static_cast<size_t>(pos) * kvd + kh * hd;
      float* vrow = vc + static_cast<size_t>(pos) * kvd + kh * hd;
      const float* vsrc = row + qd + kvd + kh * hd;
      krow[2 * j] = y0;
      krow[2 * j + 1] = y1;
      vrow[2 * j] = mri::ld_act(vsrc + 2 * j);
      vrow[2 * j + 1] = mri::ld_act(vsrc + 2 * j + 1);
    }
  }
}

// Decode attention on thread-block clusters (attention/cached.rs:141-190
// with gqa.rs:217-237): the kDecCluster CTAs of one cluster share head h, CTA
// c taking the keys [c*chunk, (c+1)*chunk) of the pos + 1 cached ones.  Each
// of its 8 warps scores rounds of 12 keys (warp w: keys base + 96 r + 12 w + i),
// a lane owning 4 head dimensions, with all of a round's K and V float4 loaded
// before any is used, and keeps an online softmax (running max, exp-sum,
// weighted V sum).  The warps' partials are combined in warp order into the
// CTA's partial in shared memory; after a cluster barrier CTA 0 reads the
// other CTAs' partials through distributed shared memory and merges them in
// rank order (no global scratch, fence or ticket), and a second cluster
// barrier keeps every CTA's shared memory alive until that read is done.
// Every CTA reaches both barriers (a CTA without keys contributes m = -inf).
constexpr int kDecCluster = 8;
constexpr int kDecWarps = 8;
constexpr int kDecRound = 8;

__global__ void __cluster_dims__(1, kDecCluster, 1) __launch_bounds__(kDecWarps * 32)
    attn_decode_cluster_kernel(const float* __restrict__ q, int n_heads, int n_kv, int hd,
                               const float* __restrict__ kc, const float* __restrict__ vc,
                               const int* __restrict__ pos_dev, float scale, float* __restrict__ out) {
  pdl_trigger();
  cg::cluster_group cluster = cg::this_cluster();
  const int h = blockIdx.x;
  const int c = static_cast<int>(cluster.block_rank());
  const int kv_h = h / (n_heads / n_kv);
  const int kvd = n_kv * hd;
  {
    // The cache rows before the current position were written by earlier
    // steps: pull this CTA's share into L2 while the QKV projection in front
    // (which writes the current row) finishes.  The position may still be
    // the previous step's value here; a prefetch of the wrong rows only costs
    // bandwidth, and every prefetched row lies inside the cache.
    const int p = *reinterpret_cast<const volatile int*>(pos_dev);
    const int chunk = (p + 1 + kDecCluster - 1) / kDecCluster;
    const int a0 = c * chunk, a1 = min(p, a0 + chunk);
    for (int i = a0 * 2 + static_cast<int>(threadIdx.x); i < a1 * 2; i += blockDim.x) {
      const float* src = (i & 1 ? vc : kc) + static_cast<size_t>(i >> 1) * kvd + static_cast<size_t>(kv_h) * hd;
      mri::prefetch_l2(src, static_cast<uint32_t>(hd * sizeof(float)));
    }
  }
  pdl_wait();
  const int total = mri::ld_act(pos_dev) + 1;
  const int chunk = (total + kDecCluster - 1) / kDecCluster;
  const int j0 = c * chunk, j1 = min(total, j0 + chunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool dim_ok = lane * 4 < hd;
  const size_t base = static_cast<size_t>(kv_h) * hd + lane * 4;
  __shared__ float wm[kDecWarps], wl[kDecWarps];
  __shared__ __align__(16) float wo[kDecWarps][kMaxHeadDim];
  __shared__ __align__(16) float cpart[kMaxHeadDim + 4];  // o[hd], then m, l
  const float4 qv = dim_ok ? mri::ld_act(reinterpret_cast<const float4*>(q + h * hd + lane * 4))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
  float m = -INFINITY, l = 0.0f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k0 = j0 + warp * kDecRound; k0 < j1; k0 += kDecWarps * kDecRound) {
    float4 kk[kDecRound], vv[kDecRound];
#pragma unroll
    for (int i = 0; i < kDecRound; ++i) {
      const bool ok = dim_ok && k0 + i < j1;
      const size_t row = static_cast<size_t>(k0 + i) * kvd + base;
      kk[i] = ok ? mri::ld_act(reinterpret_cast<const float4*>(kc + row)) : make_float4(0.f, 0.f, 0.f, 0.f);
      vv[i] = ok ? mri::ld_act(reinterpret_cast<const float4*>(vc + row)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < kDecRound; ++i) {
      if (k0 + i >= j1) break;  // warp-uniform
      const float4 kv = kk[i], vw = vv[i];
      float d = __fmaf_rn(qv.x, kv.x, 0.0f);
      d = __fmaf_rn(qv.y, kv.y, d);
      d = __fmaf_rn(qv.z, kv.z, d);
      d = __fmaf_rn(qv.w, kv.w, d);
      d = mri::warp_sum_f(d);
      const float sc = __fmul_rn(d, scale);
      const float mn = fmaxf(m, sc);
      const float corr = expf(m - mn), p = expf(sc - mn);
      l = __fadd_rn(__fmul_rn(l, corr), p);
      o.x = __fmaf_rn(p, vw.x, __fmul_rn(o.x, corr));
      o.y = __fmaf_rn(p, vw.y, __fmul_rn(o.y, corr));
      o.z = __fmaf_rn(p, vw.z, __fmul_rn(o.z, corr));
      o.w = __fmaf_rn(p, vw.w, __fmul_rn(o.w, corr));
      m = mn;
    }
  }
  // The CTA's partial: warps combined in warp order (a warp without keys has
  // m = -inf, l = 0).
  if (lane == 0) {
    wm[warp] = m;
    wl[warp] = l;
  }
  if (dim_ok) reinterpret_cast<float4*>(wo[warp])[lane] = o;
  __syncthreads();
  float bm = -INFINITY;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) bm = fmaxf(bm, wm[w]);
  for (int t = threadIdx.x; t < hd; t += blockDim.x) {
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w)
      if (wm[w] != -INFINITY) acc = __fmaf_rn(wo[w][t], expf(wm[w] - bm), acc);
    cpart[t] = acc;
  }
  if (threadIdx.x == 0) {
    float bl = 0.0f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w)
      if (wm[w] != -INFINITY) bl = __fmaf_rn(wl[w], expf(wm[w] - bm), bl);
    cpart[kMaxHeadDim] = bm;
    cpart[kMaxHeadDim + 1] = bl;
  }
  cluster.sync();
  if (c == 0) {
    // Merge the cluster's partials in rank order.
    float pm[kDecCluster], pw[kDecCluster];
    float gm = -INFINITY;
#pragma unroll
    for (int r = 0; r < kDecCluster; ++r) {
      const float* pr = cluster.map_shared_rank(cpart, r);
      pm[r] = pr[kMaxHeadDim];
      gm = fmaxf(gm, pm[r]);
    }
    float gl = 0.0f;
#pragma unroll
    for (int r = 0; r < kDecCluster; ++r) {
      pw[r] = pm[r] == -INFINITY ? 0.0f : expf(pm[r] - gm);
      gl = __fmaf_rn(cluster.map_shared_rank(cpart, r)[kMaxHeadDim + 1], pw[r], gl);
    }
    const float inv = __fdiv_rn(1.0f, gl);
    for (int t = threadIdx.x; t < hd; t += blockDim.x) {
      float acc = 0.0f;
#pragma unroll
      for (int r = 0; r < kDecCluster; ++r) acc = __fmaf_rn(cluster.map_shared_rank(cpart, r)[t], pw[r], acc);
      out[h * hd + t] = acc * inv;
    }
  }
  cluster.sync();
}

// Prefill attention (gqa.rs:217-237 with mask.rs:77-115): block (h, qb)
// handles queries [qb*16, qb*16+16) at absolute positions start + i against
// cached keys [0, start + i], online softmax over 64-key tiles in shared memory.
__global__ void __launch_bounds__(256) attn_prefill_kernel(const float* __restrict__ qkv, int ld,
                                                           int n_heads, int n_kv, int hd, int M,
                                                           int start, const float* __restrict__ kc,
                                                           const float* __restrict__ vc, float scale,
                                                           float* __restrict__ out, int out_ld) {
  extern __shared__ float sm[];
  float* sk = sm;                                   // [64][hd+1]
  float* sv = sk + kPrefillKT * (kMaxHeadDim + 1);  // [64][hd]
  float* sq = sv + kPrefillKT * kMaxHeadDim;        // [16][hd]
  const int h = blockIdx.x, q0 = blockIdx.y * kPrefillQ;
  const int kv_h = h / (n_heads / n_kv);
  const int kvd = n_kv * hd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = threadIdx.x; t < kPrefillQ * hd; t += blockDim.x) {
    const int qi = t / hd, d = t % hd;
    sq[t] = q0 + qi < M ? qkv[static_cast<size_t>(q0 + qi) * ld + h * hd + d] : 0.0f;
  }
  // Each warp owns two queries; each lane keeps hd/32 output dims per query.
  const int qa = q0 + warp * 2, qb = qa + 1;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
  float o_a[kMaxHeadDim / 32], o_b[kMaxHeadDim / 32];
#pragma unroll
  for (int i = 0; i < kMaxHeadDim / 32; ++i) o_a[i] = o_b[i] = 0.0f;
  const int last_key = start + min(q0 + kPrefillQ, M) - 1;
  for (int kt = 0; kt <= last_key; kt += kPrefillKT) {
    __syncthreads();
    const int nk = min(kPrefillKT, last_key + 1 - kt);
    for (int t = threadIdx.x; t < nk * hd; t += blockDim.x) {
      const int j = t / hd, d = t % hd;
      sk[j * (kMaxHeadDim + 1) + d] = kc[static_cast<size_t>(kt + j) * kvd + kv_h * hd + d];
      sv[j * kMaxHeadDim + d] = vc[static_cast<size_t>(kt + j) * kvd + kv_h * hd + d];
    }
    __syncthreads();
    // Lane handles keys kt+lane and kt+lane+32 for both queries.
    float s[2][2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int j = lane + 32 * r;
      float da = 0.0f, db = 0.0f;
      if (j < nk) {
        for (int d = 0; d < hd; ++d) {
          const float kv = sk[j * (kMaxHeadDim + 1) + d];
          da = __fmaf_rn(sq[(warp * 2) * hd + d], kv, da);
          db = __fmaf_rn(sq[(warp * 2 + 1) * hd + d], kv, db);
        }
      }
      const int key = kt + j;
      s[0][r] = (j < nk && qa < M && key <= start + qa) ? __fmul_rn(da, scale) : -INFINITY;
      s[1][r] = (j < nk && qb < M && key <= start + qb) ? __fmul_rn(db, scale) : -INFINITY;
    }
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
      float& m = qq ? m_b : m_a;
      float& l = qq ? l_b : l_a;
      float* o = qq ? o_b : o_a;
      float tmax = mri::warp_max(fmaxf(s[qq][0], s[qq][1]));
      const float mnew = fmaxf(m, tmax);
      if (mnew == -INFINITY) continue;  // nothing visible yet
      const float corr = expf(m - mnew);
      const float p0 = expf(s[qq][0] - mnew), p1 = expf(s[qq][1] - mnew);
      l = l * corr + mri::warp_sum_f(p0 + p1);
#pragma unroll
      for (int i = 0; i < kMaxHeadDim / 32; ++i) o[i] *= corr;
      for (int j = 0; j < nk; ++j) {
        const float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
#pragma unroll
        for (int i = 0; i < kMaxHeadDim / 32; ++i) {
          const int d = lane + 32 * i;
          if (d < hd) o[i] = __fmaf_rn(pj, sv[j * kMaxHeadDim + d], o[i]);
        }
      }
      m = mnew;
    }
  }
#pragma unroll
  for (int qq = 0; qq < 2; ++qq) {
    const int qi = qq ? qb : qa;
    if (qi >= M) continue;
    const float inv = __fdiv_rn(1.0f, qq ? l_b : l_a);
    const float* o = qq ? o_b : o_a;
#pragma unroll
    for (int i = 0; i < kMaxHeadDim / 32; ++i) {
      const int d = lane + 32 * i;
      if (d < hd) out[static_cast<size_t>(qi) * out_ld + h * hd + d] = o[i] * inv;
    }
  }
}

// Prefill attention on the tensor cores (flash-attention style): block (h, qb)
// handles queries [qb*128, qb*128+128) of head h, a warp 16 of them.  Per tile of
// 64 cached keys, S = Q K^T and O += P V run on mma.sync m16n8k16 with f16
// operands and f32 accumulators: Q is held as A fragments, K and V^T are
// converted into shared memory (rows padded so a fragment load hits 32
// banks), P comes straight from S's accumulator layout.  Every operand is
// split into f16 hi + lo parts and each product is hi.hi + hi.lo + lo.hi
// (about 22 significant bits, close to the f32 kernel): the attention output
// is quantized to int8 by the next projection, and an error of ~1e-3 (single
// f16 operands) flips enough of those roundings to move the logits by a few
// percent of their range.  The causal mask (key <= start + query), the scale
// and the online softmax (running max, sum) are f32, per row over the 4
// threads that hold it.  HD = head dim (64 or 128).  q, k and v must lie
// within the f16 range: a block that loads a value beyond it (or a NaN) sets
// *range_flag, and the host runs the call again on the f32 CUDA-core kernel.
constexpr int kFaQ = 128;  // queries per block (a warp per 16): each K/V tile is converted once per 128 queries
constexpr int kFaThreads = 2 * kFaQ;
constexpr int kFaKT = 64;  // keys per tile

__device__ __forceinline__ uint32_t half2_bits(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// True when either value is NaN or beyond the largest finite f16 (65504):
// its f16 hi part would be infinite.
__device__ __forceinline__ bool beyond_f16(float2 v) {
  return !(fabsf(v.x) <= 65504.0f) | !(fabsf(v.y) <= 65504.0f);
}

// Two floats as f16 pairs hi = f16(x), lo = f16(x - hi).
__device__ __forceinline__ void split_half2(float2 v, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(v.x, v.y);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = half2_bits(__fsub_rn(v.x, hf.x), __fsub_rn(v.y, hf.y));
}

__device__ __forceinline__ void mma_f16_m16n8k16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int HD>
__global__ void __launch_bounds__(kFaThreads) attn_prefill_tc_kernel(const float* __restrict__ qkv, int ld,
                                                              int n_heads, int n_kv, int M, int start,
                                                              const float* __restrict__ kc,
                                                              const float* __restrict__ vc, float scale,
                                                              float* __restrict__ out, int out_ld,
                                                              float* __restrict__ part,
                                                              int* __restrict__ tickets, int split_min,
                                                              int* __restrict__ range_flag) {
  constexpr int KS = HD / 16;     // k steps of S = Q K^T
  constexpr int NT = HD / 8;      // n tiles of O
  constexpr int SK = HD + 8;      // halves per K row in shared memory
  constexpr int SV = kFaKT + 8;   // halves per V^T row (one head dim) in shared memory
  extern __shared__ __align__(16) __half fa_smem[];
  __half* sK = fa_smem;                 // [64 keys][SK] hi parts
  __half* sKl = sK + kFaKT * SK;        // [64 keys][SK] lo parts
  __half* sVt = sKl + kFaKT * SK;       // [HD][SV] hi parts
  __half* sVtl = sVt + HD * SV;         // [HD][SV] lo parts
  // blockIdx.y = (query block, split), the longest walks (last query
  // blocks) first so that the short ones fill in behind them.
  const int splits_grid = split_min > 0 ? 2 : 1;
  const int n_qb = static_cast<int>(gridDim.y) / splits_grid;
  const int qb = n_qb - 1 - static_cast<int>(blockIdx.y) / splits_grid;
  const int split = static_cast<int>(blockIdx.y) % splits_grid;
  const int h = blockIdx.x, q0 = qb * kFaQ;
  const int kv_h = h / (n_heads / n_kv);
  const int kvd = n_kv * HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int ra = q0 + warp * 16 + g, rb = ra + 8;  // this thread's two query rows
  // Q fragments (rows ra, rb; dims 16k + 2t, +1 and 16k + 8 + 2t, +1), hi and lo.
  uint32_t qa[KS][4], ql[KS][4];
  bool bad = false;  // a q, k or v value this thread converted lies beyond the f16 range
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    const int d0 = 16 * k + 2 * t;
    float2 a = make_float2(0.f, 0.f), b = a, c = a, e = a;
    if (ra < M) {
      const float* q = qkv + static_cast<size_t>(ra) * ld + h * HD;
      a = *reinterpret_cast<const float2*>(q + d0);
      c = *reinterpret_cast<const float2*>(q + d0 + 8);
    }
    if (rb < M) {
      const float* q = qkv + static_cast<size_t>(rb) * ld + h * HD;
      b = *reinterpret_cast<const float2*>(q + d0);
      e = *reinterpret_cast<const float2*>(q + d0 + 8);
    }
    bad |= beyond_f16(a) | beyond_f16(b) | beyond_f16(c) | beyond_f16(e);
    split_half2(a, qa[k][0], ql[k][0]);
    split_half2(b, qa[k][1], ql[k][1]);
    split_half2(c, qa[k][2], ql[k][2]);
    split_half2(e, qa[k][3], ql[k][3]);
  }
  if (bad) *reinterpret_cast<volatile int*>(range_flag) = 1;
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
  const int last_key = start + min(q0 + kFaQ, M) - 1;
  // Key tiles [t0, t1) of this block.  The causal prefix of the last query
  // blocks is the longest walk; from split_min tiles on it goes to two
  // blocks (split 0 and 1) whose partial results the later one merges.
  const int n_tiles = last_key / kFaKT + 1;
  const int n_splits = split_min > 0 && n_tiles >= split_min ? 2 : 1;
  if (split >= n_splits) return;
  const int t0 = split * n_tiles / n_splits, t1 = (split + 1) * n_tiles / n_splits;
  for (int kt = t0 * kFaKT; kt < t1 * kFaKT; kt += kFaKT) {
    const int nk = min(kFaKT, last_key + 1 - kt);
    __syncthreads();
    // K tile -> sK[key][dim], V tile -> sVt[dim][key] (f16); keys past nk are 0.
    for (int i = threadIdx.x; i < kFaKT * (HD / 4); i += blockDim.x) {
      const int j = i / (HD / 4), d = (i % (HD / 4)) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (j < nk) {
        const size_t off = static_cast<size_t>(kt + j) * kvd + kv_h * HD + d;
        kv = *reinterpret_cast<const float4*>(kc + off);
        vv = *reinterpret_cast<const float4*>(vc + off);
        bad |= beyond_f16(make_float2(kv.x, kv.y)) | beyond_f16(make_float2(kv.z, kv.w)) |
               beyond_f16(make_float2(vv.x, vv.y)) | beyond_f16(make_float2(vv.z, vv.w));
      }
      uint32_t h0, l0, h1, l1;
      split_half2(make_float2(kv.x, kv.y), h0, l0);
      split_half2(make_float2(kv.z, kv.w), h1, l1);
      *reinterpret_cast<uint2*>(sK + j * SK + d) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(sKl + j * SK + d) = make_uint2(l0, l1);
      const float vf[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half hv = __float2half_rn(vf[i]);
        sVt[(d + i) * SV + j] = hv;
        sVtl[(d + i) * SV + j] = __float2half_rn(__fsub_rn(vf[i], __half2float(hv)));
      }
    }
    __syncthreads();
    // A tile every key of which lies past this warp's last query is masked
    // for all of its rows: skip its MMAs (warp-uniform; the loads above are
    // shared by the block and stay).
    if (kt > start + q0 + warp * 16 + 15) continue;
    // S = Q K^T for this warp's 16 queries x 64 keys (8 n tiles of 8 keys).
    float sc[kFaKT / 8][4];
#pragma unroll
    for (int n = 0; n < kFaKT / 8; ++n) {
      sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
      const __half* kr = sK + (n * 8 + g) * SK + 2 * t;
      const __half* klr = sKl + (n * 8 + g) * SK + 2 * t;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        const uint32_t kh0 = *reinterpret_cast<const uint32_t*>(kr + 16 * k);
        const uint32_t kh1 = *reinterpret_cast<const uint32_t*>(kr + 16 * k + 8);
        mma_f16_m16n8k16(sc[n], qa[k], kh0, kh1);
        mma_f16_m16n8k16(sc[n], ql[k], kh0, kh1);
        mma_f16_m16n8k16(sc[n], qa[k], *reinterpret_cast<const uint32_t*>(klr + 16 * k),
                         *reinterpret_cast<const uint32_t*>(klr + 16 * k + 8));
      }
    }
    // Scale and causal mask; row maxima over the 4 threads of a row.
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int n = 0; n < kFaKT / 8; ++n) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int key = kt + n * 8 + 2 * t + (c & 1);
        const int row = c < 2 ? ra : rb;
        const bool ok = key - kt < nk && row < M && key <= start + row;
        sc[n][c] = ok ? __fmul_rn(sc[n][c], scale) : -INFINITY;
      }
      mx_a = fmaxf(mx_a, fmaxf(sc[n][0], sc[n][1]));
      mx_b = fmaxf(mx_b, fmaxf(sc[n][2], sc[n][3]));
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    // A row with nothing visible yet keeps m = -inf, l = 0, o = 0.
    const float corr_a = mn_a == -INFINITY ? 1.0f : expf(m_a - mn_a);
    const float corr_b = mn_b == -INFINITY ? 1.0f : expf(m_b - mn_b);
    float ps_a = 0.0f, ps_b = 0.0f;
#pragma unroll
    for (int n = 0; n < kFaKT / 8; ++n) {
      sc[n][0] = sc[n][0] == -INFINITY ? 0.0f : expf(sc[n][0] - mn_a);
      sc[n][1] = sc[n][1] == -INFINITY ? 0.0f : expf(sc[n][1] - mn_a);
      sc[n][2] = sc[n][2] == -INFINITY ? 0.0f : expf(sc[n][2] - mn_b);
      sc[n][3] = sc[n][3] == -INFINITY ? 0.0f : expf(sc[n][3] - mn_b);
      ps_a += sc[n][0] + sc[n][1];
      ps_b += sc[n][2] + sc[n][3];
    }
    l_a = l_a * corr_a + ps_a;
    l_b = l_b * corr_b + ps_b;
    m_a = mn_a;
    m_b = mn_b;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= corr_a;
      o[n][1] *= corr_a;
      o[n][2] *= corr_b;
      o[n][3] *= corr_b;
    }
    // O += P V: P's k step j (keys 16j..16j+15) is S's n tiles 2j and 2j+1.
#pragma unroll
    for (int j = 0; j < kFaKT / 16; ++j) {
      uint32_t pa[4], pl[4];
      split_half2(make_float2(sc[2 * j][0], sc[2 * j][1]), pa[0], pl[0]);
      split_half2(make_float2(sc[2 * j][2], sc[2 * j][3]), pa[1], pl[1]);
      split_half2(make_float2(sc[2 * j + 1][0], sc[2 * j + 1][1]), pa[2], pl[2]);
      split_half2(make_float2(sc[2 * j + 1][2], sc[2 * j + 1][3]), pa[3], pl[3]);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const __half* vr = sVt + (n * 8 + g) * SV + 16 * j + 2 * t;
        const __half* vlr = sVtl + (n * 8 + g) * SV + 16 * j + 2 * t;
        const uint32_t vh0 = *reinterpret_cast<const uint32_t*>(vr);
        const uint32_t vh1 = *reinterpret_cast<const uint32_t*>(vr + 8);
        mma_f16_m16n8k16(o[n], pa, vh0, vh1);
        mma_f16_m16n8k16(o[n], pl, vh0, vh1);
        mma_f16_m16n8k16(o[n], pa, *reinterpret_cast<const uint32_t*>(vlr),
                         *reinterpret_cast<const uint32_t*>(vlr + 8));
      }
    }
  }
  if (bad) *reinterpret_cast<volatile int*>(range_flag) = 1;
  // Row sums over the 4 threads of a row, then O / l.
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  if (n_splits > 1) {
    // Both splits store (o, m, l) of their 128 rows; the block that arrives
    // second merges the two records in split order (the same sums whichever
    // finishes first) and resets the ticket for the next launch.
    constexpr int kRec = kFaQ * (HD + 2);
    const int pair = qb * gridDim.x + h;
    float* rec = part + (static_cast<size_t>(pair) * 2 + split) * kRec;
    const int la = warp * 16 + g, lb = la + 8;  // local rows
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int d = n * 8 + 2 * t;
      *reinterpret_cast<float2*>(rec + la * HD + d) = make_float2(o[n][0], o[n][1]);
      *reinterpret_cast<float2*>(rec + lb * HD + d) = make_float2(o[n][2], o[n][3]);
    }
    if (t == 0) {
      rec[kFaQ * HD + la] = m_a;
      rec[kFaQ * HD + lb] = m_b;
      rec[kFaQ * HD + kFaQ + la] = l_a;
      rec[kFaQ * HD + kFaQ + lb] = l_b;
    }
    __threadfence();
    __syncthreads();
    __shared__ int fa_last;
    if (threadIdx.x == 0) fa_last = atomicAdd(tickets + pair, 1) == 1;
    __syncthreads();
    if (!fa_last) return;
    __threadfence();
    if (threadIdx.x == 0) tickets[pair] = 0;
    const float* r0 = part + static_cast<size_t>(pair) * 2 * kRec;
    const float* r1 = r0 + kRec;
    const float m0a = __ldcg(r0 + kFaQ * HD + la), m1a = __ldcg(r1 + kFaQ * HD + la);
    const float m0b = __ldcg(r0 + kFaQ * HD + lb), m1b = __ldcg(r1 + kFaQ * HD + lb);
    const float mxa = fmaxf(m0a, m1a), mxb = fmaxf(m0b, m1b);
    // A split that saw no key of a row (m = -inf) contributes nothing.
    const float c0a = m0a == -INFINITY ? 0.0f : expf(m0a - mxa);
    const float c1a = m1a == -INFINITY ? 0.0f : expf(m1a - mxa);
    const float c0b = m0b == -INFINITY ? 0.0f : expf(m0b - mxb);
    const float c1b = m1b == -INFINITY ? 0.0f : expf(m1b - mxb);
    l_a = __fadd_rn(__fmul_rn(__ldcg(r0 + kFaQ * HD + kFaQ + la), c0a),
                    __fmul_rn(__ldcg(r1 + kFaQ * HD + kFaQ + la), c1a));
    l_b = __fadd_rn(__fmul_rn(__ldcg(r0 + kFaQ * HD + kFaQ + lb), c0b),
                    __fmul_rn(__ldcg(r1 + kFaQ * HD + kFaQ + lb), c1b));
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int d = n * 8 + 2 * t;
      const float2 p0a = __ldcg(reinterpret_cast<const float2*>(r0 + la * HD + d));
      const float2 p1a = __ldcg(reinterpret_cast<const float2*>(r1 + la * HD + d));
      const float2 p0b = __ldcg(reinterpret_cast<const float2*>(r0 + lb * HD + d));
      const float2 p1b = __ldcg(reinterpret_cast<const float2*>(r1 + lb * HD + d));
      o[n][0] = __fadd_rn(__fmul_rn(p0a.x, c0a), __fmul_rn(p1a.x, c1a));
      o[n][1] = __fadd_rn(__fmul_rn(p0a.y, c0a), __fmul_rn(p1a.y, c1a));
      o[n][2] = __fadd_rn(__fmul_rn(p0b.x, c0b), __fmul_rn(p1b.x, c1b));
      o[n][3] = __fadd_rn(__fmul_rn(p0b.y, c0b), __fmul_rn(p1b.y, c1b));
    }
  }
  const float ia = __fdiv_rn(1.0f, l_a), ib = __fdiv_rn(1.0f, l_b);
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int d = n * 8 + 2 * t;
    if (ra < M)
      *reinterpret_cast<float2*>(out + static_cast<size_t>(ra) * out_ld + h * HD + d) =
          make_float2(o[n][0] * ia, o[n][1] * ia);
    if (rb < M)
      *reinterpret_cast<float2*>(out + static_cast<size_t>(rb) * out_ld + h * HD + d) =
          make_float2(o[n][2] * ib, o[n][3] * ib);
  }
}

// Dynamic shared memory of attn_prefill_tc_kernel<hd>: K and V^T tiles, hi and lo.
size_t fa_smem_bytes(int hd) {
  return (2 * static_cast<size_t>(kFaKT) * (hd + 8) + 2 * static_cast<size_t>(hd) * (kFaKT + 8)) *
         sizeof(__half);
}

// Greedy sampling: argmax (first index on ties; NaN never wins) -> next
// token; position += 1.  Block b reduces a slice of the logits into
// part[b]; the last block to finish (ticket) reduces the partials, writes the
// token to *token and gen[*pos + 1], advances *pos and resets the ticket.
constexpr int kArgmaxBlocks = 32;

__device__ __forceinline__ void better(float& best, int& idx, float v, int i) {
  if (v > best || (v == best && i < idx)) {
    best = v;
    idx = i;
  }
}

__device__ __forceinline__ void block_argmax(float& best, int& idx, float* sb, int* si) {
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    better(best, idx, ob, oi);
  }
  if ((threadIdx.x & 31) == 0) {
    sb[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) better(best, idx, sb[w], si[w]);
}

__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ logits, int V,
                                                     float* __restrict__ part_v,
                                                     int* __restrict__ part_i, int* __restrict__ ticket,
                                                     uint32_t* __restrict__ token,
                                                     int* __restrict__ pos,
                                                     uint32_t* __restrict__ gen) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sb[8];
  __shared__ int si[8];
  __shared__ int last;
  // Block ranges of a multiple of 4 logits, read in 16-byte pieces (the
  // order of the comparisons does not matter: `better` is a total order on
  // (value, -index) that never picks a NaN).
  const int per = ((V + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x) + 3) & ~3;
  const int lo = min(V, static_cast<int>(blockIdx.x) * per), hi = min(V, lo + per);
  float best = -INFINITY;
  int idx = 0x7fffffff;
  const int hi4 = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 ? lo + ((hi - lo) & ~3) : lo;
  for (int i = lo + 4 * static_cast<int>(threadIdx.x); i < hi4; i += 4 * static_cast<int>(blockDim.x)) {
    const float4 v = mri::ld_act(reinterpret_cast<const float4*>(logits + i));
    better(best, idx, v.x, i);
    better(best, idx, v.y, i + 1);
    better(best, idx, v.z, i + 2);
    better(best, idx, v.w, i + 3);
  }
  for (int i = hi4 + threadIdx.x; i < hi; i += blockDim.x) better(best, idx, mri::ld_act(logits + i), i);
  block_argmax(best, idx, sb, si);
  if (threadIdx.x == 0) {
    part_v[blockIdx.x] = best;
    part_i[blockIdx.x] = idx;
    __threadfence();
    last = atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  best = -INFINITY;
  idx = 0x7fffffff;
  for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += blockDim.x)
    better(best, idx, __ldcg(part_v + b), __ldcg(part_i + b));
  __syncthreads();
  block_argmax(best, idx, sb, si);
  if (threadIdx.x == 0) {
    const uint32_t t = static_cast<uint32_t>(idx == 0x7fffffff ? 0 : idx);
    const int p = mri::ld_act(pos);
    *token = t;
    gen[p + 1] = t;  // the token generated for position pos + 1
    *pos = p + 1;
    *ticket = 0;
  }
}

// Synthetic weights for benchmarking: int8 uniform in [-127, 127] and scales
// uniform in [lo, hi] from a counter-based hash (splitmix64).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void fill_i8_kernel(int8_t* __restrict__ w, size_t n, uint64_t seed) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    w[i] = static_cast<int8_t>(static_cast<int>(mix64(seed ^ (i * 0xD1B54A32D192ED03ull)) % 255u) - 127);
}

__global__ void fill_f32_kernel(float* __restrict__ w, size_t n, uint64_t seed, float lo, float hi) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float u = static_cast<float>(mix64(seed ^ (i * 0xA24BAED4963EE407ull)) >> 40) * (1.0f / 16777216.0f);
    w[i] = lo + (hi - lo) * u;
  }
}

thread_local std::string g_model_error;

int fail(int code, const char* fmt, ...) {
  char buf[400];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_model_error = buf;
  return code;
}

#define LL_TRY(expr)                                                              \
  do {                                                                            \
    cudaError_t _e = (expr);                                                      \
    if (_e != cudaSuccess) return fail(MRI_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

#define LL_RC(expr)                                         \
  do {                                                      \
    int _rc = (expr);                                       \
    if (_rc != MRI_OK) return fail(_rc, "%s", mri_last_error()); \
  } while (0)

}  // namespace

struct mri_llama {
  mri_ctx* ctx = nullptr;
  mri_llama_config cfg{};
  int hd = 0, qd = 0, kvd = 0, qkv_w = 0;
  size_t max_tokens = 0;
  // weights
  float* embd = nullptr;
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  float* out_norm = nullptr;
  int8_t* w_blob = nullptr;  // all int8 projection weights
  float* s_blob = nullptr;   // all per-channel scales
  std::vector<mri_qmatrix> wqkv, wo, wgu, wdown;
  mri_qmatrix wout{};
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  // cache and activations
  float *kc = nullptr, *vc = nullptr;
  float *x = nullptr, *qkv = nullptr, *attn = nullptr, *gu = nullptr;
  float* logits = nullptr;
  int* tickets = nullptr;      // the greedy argmax's ticket counter
  float* fa_part = nullptr;    // prefill attention: two split records per (query block, head)
  int* fa_tickets = nullptr;   // prefill attention: split counters per (query block, head)
  int* fa_range = nullptr;     // prefill attention: set when q, k or v lay beyond the f16 range
  bool cuda_core_attn = false; // rerun after such a call: prefill attention on the f32 CUDA-core kernel
  size_t attn_fallbacks = 0;   // calls rerun that way
  float* amax_v = nullptr;     // argmax partials
  int* amax_i = nullptr;
  bool fused_decode = false;   // decode projections carry the RoPE/KV and SwiGLU epilogues
  uint32_t* d_tokens = nullptr;
  uint32_t* d_gen = nullptr;  // [max_seq + 1] tokens produced by greedy argmax
  int* d_pos = nullptr;
  cudaGraphExec_t decode_exec = nullptr;
  size_t graph_kernels = 0;
  std::vector<void*> allocs;
};

namespace {

template <typename T>
int dalloc(mri_llama* m, T** p, size_t count) {
  void* v = nullptr;
  LL_TRY(cudaMalloc(&v, std::max<size_t>(count * sizeof(T), 256)));
  m->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return MRI_OK;
}

// Layout of the weight blobs: per layer [wqkv | wo | wgu | wdown], then the
// LM head.  Offsets in elements.
struct BlobLayout {
  size_t per_layer_w, per_layer_s, total_w, total_s;
  size_t qkv_w, o_w, gu_w, down_w;
};

BlobLayout blob_layout(const mri_llama* m) {
  const auto& c = m->cfg;
  BlobLayout b{};
  b.qkv_w = static_cast<size_t>(m->qkv_w) * c.dim;
  b.o_w = static_cast<size_t>(c.dim) * m->qd;
  b.gu_w = static_cast<size_t>(2) * c.ffn_dim * c.dim;
  b.down_w = static_cast<size_t>(c.dim) * c.ffn_dim;
  b.per_layer_w = b.qkv_w + b.o_w + b.gu_w + b.down_w;
  b.per_layer_s = static_cast<size_t>(m->qkv_w) + c.dim + 2 * c.ffn_dim + c.dim;
  // Every matrix is padded to 256 bytes (weights) / 64 floats (scales).
  auto pw = [](size_t v) { return (v + 255) / 256 * 256; };
  auto ps = [](size_t v) { return (v + 63) / 64 * 64; };
  b.per_layer_w = pw(b.qkv_w) + pw(b.o_w) + pw(b.gu_w) + pw(b.down_w);
  b.per_layer_s = ps(m->qkv_w) + ps(c.dim) + ps(2 * static_cast<size_t>(c.ffn_dim)) + ps(c.dim);
  b.total_w = b.per_layer_w * c.n_layers + pw(static_cast<size_t>(c.vocab) * c.dim);
  b.total_s = b.per_layer_s * c.n_layers + ps(c.vocab);
  return b;
}

// Launch with programmatic stream serialization (see the glue-kernel note).
template <typename... KArgs, typename... Args>
cudaError_t pdl_launch(const mri_llama* m, void (*k)(KArgs...), dim3 grid, dim3 block, cudaStream_t st,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = m->ctx->dev.opt.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// One INT8 projection with per-tensor quantization of x [rows, k], with the
// producer op fused in front (RMSNorm weight `norm`, or SwiGLU over [gate|up]
// rows) and the residual add fused behind (out = residual + product).
int proj(mri_llama* m, const float* x, size_t rows, const mri_qmatrix& w, float* out,
         const float* norm = nullptr, int swiglu = 0, const float* residual = nullptr,
         const mri::EpiArgs* epi = nullptr, int pre_stages = -1) {
  LL_RC(mri::matmul_int8_fused(m->ctx, x, rows, w.k_in, norm, m->cfg.rms_eps, swiglu, &w, residual,
                               out, epi, pre_stages));
  return MRI_OK;
}

// Runs the blocks for `rows` tokens already embedded in m->x, at absolute
// positions [pos0, pos0+rows) (or *d_pos when decode_dev).  Per block:
//   qkv = proj(rmsnorm(x, attn_norm))        (forward_int8.rs:361-372)
//   rope + cache write; attention
//   x   = x + proj(attn, wo)                 (:374-393)
//   x   = x + proj(swiglu(proj(rmsnorm(x, ffn_norm), wgu)), wdown)  (:395-402)
// The gate/up rows of wgu are interleaved.  In the fused decode step the RoPE
// rotation, the cache write and the SwiGLU run in the projections' epilogues.
// Layers [l_begin, l_end) (all by default) on the residual stream m->x.
int run_blocks(mri_llama* m, size_t rows, int pos0, bool decode_dev, uint32_t l_begin = 0,
               uint32_t l_end = ~0u) {
  const auto& c = m->cfg;
  cudaStream_t st = m->ctx->stream;
  const float scale = 1.0f / std::sqrt(static_cast<float>(m->hd));
  const size_t layer_kv = static_cast<size_t>(c.max_seq) * m->kvd;
  const bool fused = decode_dev && m->fused_decode;
  for (uint32_t l = l_begin; l < std::min(l_end, c.n_layers); ++l) {
    float* kc = m->kc + l * layer_kv;
    float* vc = m->vc + l * layer_kv;
    if (fused) {
      mri::EpiArgs e;
      e.mode = mri::EPI_ROPE_KV;
      e.pos_dev = m->d_pos;
      e.cos_t = m->rope_cos;
      e.sin_t = m->rope_sin;
      e.hd = m->hd;
      e.qd = m->qd;
      e.kvd = m->kvd;
      e.kc = kc;
      e.vc = vc;
      if (int rc = proj(m, m->x, rows, m->wqkv[l], m->qkv, m->attn_norm + l * c.dim, 0, nullptr, &e))
        return rc;
    } else {
      if (int rc = proj(m, m->x, rows, m->wqkv[l], m->qkv, m->attn_norm + l * c.dim)) return rc;
      if (!decode_dev && m->hd % 4 == 0 && m->qkv_w % 4 == 0) {
        LL_TRY(pdl_launch(m, rope_kv_rows_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), st, m->qkv,
                          m->qkv_w, c.n_heads, c.n_kv_heads, m->hd, m->rope_cos, m->rope_sin, pos0, kc, vc));
      } else {
        LL_TRY(pdl_launch(m, rope_kv_kernel, dim3(static_cast<unsigned>(rows), c.n_heads + c.n_kv_heads),
                          dim3(64), st, m->qkv, m->qkv_w, c.n_heads, c.n_kv_heads, m->hd, m->rope_cos,
                          m->rope_sin, pos0, decode_dev ? m->d_pos : nullptr, kc, vc));
      }
    }
    if (decode_dev) {
      LL_TRY(pdl_launch(m, attn_decode_cluster_kernel, dim3(c.n_heads, kDecCluster), dim3(kDecWarps * 32), st,
                        m->qkv, c.n_heads, c.n_kv_heads, m->hd, kc, vc, m->d_pos, scale, m->attn));
    } else if ((m->hd == 64 || m->hd == 128) && (m->qkv_w % 2) == 0 && (m->qd % 2) == 0 &&
               m->ctx->dev.opt.tc_attn && !m->cuda_core_attn) {
      // Key tiles from which a query block's walk is split over two blocks (0 = never).
      const int split_min = std::max(0, m->ctx->dev.opt.fa_split);
      const dim3 grid(c.n_heads, static_cast<unsigned>((rows + kFaQ - 1) / kFaQ) * (split_min > 0 ? 2 : 1));
      const size_t smem = fa_smem_bytes(m->hd);
      static bool fa_attr_set[64] = {false};
      const int dv = m->ctx->device;
      if (dv >= 0 && dv < 64 && !fa_attr_set[dv]) {
        LL_TRY(cudaFuncSetAttribute(attn_prefill_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(fa_smem_bytes(64))));
        LL_TRY(cudaFuncSetAttribute(attn_prefill_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(fa_smem_bytes(128))));
        fa_attr_set[dv] = true;
      }
      if (m->hd == 64)
        attn_prefill_tc_kernel<64><<<grid, kFaThreads, smem, st>>>(m->qkv, m->qkv_w, c.n_heads, c.n_kv_heads,
                                                            static_cast<int>(rows), pos0, kc, vc, scale,
                                                            m->attn, m->qd, m->fa_part, m->fa_tickets,
                                                            split_min, m->fa_range);
      else
        attn_prefill_tc_kernel<128><<<grid, kFaThreads, smem, st>>>(m->qkv, m->qkv_w, c.n_heads, c.n_kv_heads,
                                                             static_cast<int>(rows), pos0, kc, vc, scale,
                                                             m->attn, m->qd, m->fa_part, m->fa_tickets,
                                                             split_min, m->fa_range);
    } else {
      const size_t smem = (kPrefillKT * (kMaxHeadDim + 1) + kPrefillKT * kMaxHeadDim +
                           kPrefillQ * kMaxHeadDim) * sizeof(float);
      static bool attr_set[64] = {false};
      const int dv = m->ctx->device;
      if (dv >= 0 && dv < 64 && !attr_set[dv]) {
        LL_TRY(cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
        attr_set[dv] = true;
      }
      attn_prefill_kernel<<<dim3(c.n_heads, static_cast<unsigned>((rows + kPrefillQ - 1) / kPrefillQ)),
                            256, smem, st>>>(m->qkv, m->qkv_w, c.n_heads, c.n_kv_heads, m->hd,
                                             static_cast<int>(rows), pos0, kc, vc, scale, m->attn,
                                             m->qd);
    }
    // The O projection follows attention, which leaves HBM mostly idle: in
    // the decode step its producer fills the whole ring while attention runs.
    if (int rc = proj(m, m->attn, rows, m->wo[l], m->x, nullptr, 0, m->x, nullptr, decode_dev ? 1 << 20 : -1))
      return rc;
    if (fused) {
      mri::EpiArgs e;
      e.mode = mri::EPI_SWIGLU;
      if (int rc = proj(m, m->x, rows, m->wgu[l], m->gu, m->ffn_norm + l * c.dim, 0, nullptr, &e)) return rc;
      if (int rc = proj(m, m->gu, rows, m->wdown[l], m->x, nullptr, 0, m->x)) return rc;
    } else {
      if (int rc = proj(m, m->x, rows, m->wgu[l], m->gu, m->ffn_norm + l * c.dim)) return rc;
      if (int rc = proj(m, m->gu, rows, m->wdown[l], m->x, nullptr, 1, m->x)) return rc;
    }
  }
  LL_TRY(cudaGetLastError());
  return MRI_OK;
}

// Logits for rows [first, first+count) of m->x: output RMSNorm fused into the
// LM-head projection (forward_int8.rs:526-528).
int lm_head(mri_llama* m, size_t first, size_t count) {
  return proj(m, m->x + first * m->cfg.dim, count, m->wout, m->logits, m->out_norm);
}

int check_tokens(const mri_llama* m, const uint32_t* tokens, size_t n) {
  if (n == 0) return fail(MRI_ERR_INVALID_SHAPE, "forward: token list must not be empty");
  if (n > m->max_tokens)
    return fail(MRI_ERR_INVALID_SHAPE, "forward: %zu tokens exceed max_seq=%u", n, m->cfg.max_seq);
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] >= m->cfg.vocab)
      return fail(MRI_ERR_INVALID_SHAPE, "token id %u >= vocab_size %u", tokens[i], m->cfg.vocab);
  return MRI_OK;
}

// Prefill `n` host tokens at positions [pos0, pos0 + n): writes those cache
// rows and attends to cache rows [0, pos0 + n).
int prefill(mri_llama* m, const uint32_t* tokens, size_t n, size_t pos0 = 0) {
  cudaStream_t st = m->ctx->stream;
  LL_TRY(cudaMemcpyAsync(m->d_tokens, tokens, n * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
  embed_kernel<<<static_cast<unsigned>(n), 256, 0, st>>>(m->d_tokens, m->embd, m->cfg.dim, m->x);
  return run_blocks(m, n, static_cast<int>(pos0), false);
}

// After the stream has drained: true (and the flag cleared) when a prefill
// attention launch since the last check met a q, k or v value beyond the
// f16 range.  The call that made it is then run again with the prefill
// attention on the f32 CUDA-core kernel (m->cuda_core_attn), which rewrites
// every buffer and cache row the first run wrote.
bool take_range_flag(mri_llama* m) {
  int v = 0;
  if (cudaMemcpy(&v, m->fa_range, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess || v == 0) return false;
  cudaMemset(m->fa_range, 0, sizeof(int));
  return true;
}

// Prefill of `n` tokens at pos0 with logits of every row copied to the host
// (LlamaModelInt8::forward at pos0 = 0; the block loop of
// forward_cached_parallel at pos0 > 0).
int forward_rows(mri_llama* m, const uint32_t* tokens, size_t n, size_t pos0, float* logits) {
  for (int attempt = 0;; ++attempt) {
    if (int rc = prefill(m, tokens, n, pos0)) return rc;
    if (int rc = lm_head(m, 0, n)) return rc;
    if (logits)
      LL_TRY(cudaMemcpyAsync(logits, m->logits, n * m->cfg.vocab * 4, cudaMemcpyDeviceToHost,
                             m->ctx->stream));
    LL_TRY(cudaStreamSynchronize(m->ctx->stream));
    const bool redo = attempt == 0 && take_range_flag(m);
    m->cuda_core_attn = redo;
    if (!redo) break;
    m->attn_fallbacks++;
  }
  return mri_ctx_check_device_status(m->ctx) ? fail(MRI_ERR_TIMEOUT, "%s", mri_last_error()) : MRI_OK;
}

int launch_argmax(mri_llama* m) {
  LL_TRY(pdl_launch(m, argmax_kernel, dim3(kArgmaxBlocks), dim3(256), m->ctx->stream, m->logits,
                    static_cast<int>(m->cfg.vocab), m->amax_v, m->amax_i, m->tickets,
                    m->d_tokens, m->d_pos, m->d_gen));
  return MRI_OK;
}

// One decode step entirely on the device: token from d_tokens[0], position
// from *d_pos; ends with argmax -> d_tokens[0] and *d_pos += 1.
int decode_step(mri_llama* m) {
  cudaStream_t st = m->ctx->stream;
  LL_TRY(pdl_launch(m, embed_kernel, dim3(1), dim3(256), st, m->d_tokens, m->embd, m->cfg.dim, m->x));
  if (int rc = run_blocks(m, 1, 0, true)) return rc;
  if (int rc = lm_head(m, 0, 1)) return rc;
  return launch_argmax(m);
}

int ensure_decode_graph(mri_llama* m) {
  if (m->decode_exec) return MRI_OK;
  cudaStream_t st = m->ctx->stream;
  // One eager step first: sizes every lazily-grown buffer and sets kernel
  // attributes, so the captured launches make no allocation.  It runs on a
  // scratch position, which the caller's next state overwrites.
  const int scratch_pos = static_cast<int>(m->cfg.max_seq) - 1;
  LL_TRY(cudaMemcpyAsync(m->d_pos, &scratch_pos, sizeof(int), cudaMemcpyHostToDevice, st));
  LL_TRY(cudaMemsetAsync(m->d_tokens, 0, sizeof(uint32_t), st));
  if (int rc = decode_step(m)) return rc;
  LL_TRY(cudaStreamSynchronize(st));
  cudaGraph_t g = nullptr;
  LL_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  const int rc = decode_step(m);
  cudaError_t e = cudaStreamEndCapture(st, &g);
  if (rc != MRI_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  LL_TRY(e);
  cudaGraphGetNodes(g, nullptr, &m->graph_kernels);
  e = cudaGraphInstantiate(&m->decode_exec, g, 0);
  cudaGraphDestroy(g);
  LL_TRY(e);
  return MRI_OK;
}

}  // namespace

extern "C" {

const char* mri_llama_last_error(void) { return g_model_error.c_str(); }

int mri_llama_create(mri_ctx* ctx, const mri_llama_config* cfg, mri_llama** out) {
  g_model_error.clear();
  if (!ctx || !cfg || !out) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  const auto& c = *cfg;
  if (c.n_layers == 0 || c.dim == 0 || c.n_heads == 0 || c.ffn_dim == 0 || c.vocab == 0 ||
      c.max_seq == 0)
    return fail(MRI_ERR_INVALID_SHAPE, "config fields must be non-zero");
  const uint32_t n_kv = c.n_kv_heads ? c.n_kv_heads : c.n_heads;
  if (c.dim % c.n_heads || c.n_heads % n_kv)
    return fail(MRI_ERR_INVALID_SHAPE, "dim %% n_heads and n_heads %% n_kv_heads must be 0");
  const int hd = static_cast<int>(c.dim / c.n_heads);
  if (hd % 8 || hd > kMaxHeadDim)
    return fail(MRI_ERR_INVALID_SHAPE, "head_dim=%d must be a multiple of 8 and <= %d", hd, kMaxHeadDim);
  cudaSetDevice(ctx->device);
  mri_llama* m = new mri_llama();
  // A private context on the caller's stream: its scratch is the model's own,
  // so products run by the caller on `ctx` cannot move it under the captured
  // decode graph.
  if (mri_ctx_create_on_stream(ctx->device, ctx->stream, &m->ctx) != MRI_OK) {
    delete m;
    return fail(MRI_ERR_CUDA, "model context: %s", mri_last_error());
  }
  m->ctx->dev.opt = ctx->dev.opt;  // the creating context's kernel-variant options
  m->cfg = c;
  m->cfg.n_kv_heads = n_kv;
  m->hd = hd;
  m->qd = static_cast<int>(c.n_heads) * hd;
  m->kvd = static_cast<int>(n_kv) * hd;
  m->qkv_w = m->qd + 2 * m->kvd;
  m->max_tokens = c.max_seq;
  const size_t T = m->max_tokens;
  const BlobLayout b = blob_layout(m);
  int rc = MRI_OK;
  rc = rc ? rc : dalloc(m, &m->embd, static_cast<size_t>(c.vocab) * c.dim);
  rc = rc ? rc : dalloc(m, &m->attn_norm, static_cast<size_t>(c.n_layers) * c.dim);
  rc = rc ? rc : dalloc(m, &m->ffn_norm, static_cast<size_t>(c.n_layers) * c.dim);
  rc = rc ? rc : dalloc(m, &m->out_norm, c.dim);
  rc = rc ? rc : dalloc(m, &m->w_blob, b.total_w + 256);
  rc = rc ? rc : dalloc(m, &m->s_blob, b.total_s + 64);
  rc = rc ? rc : dalloc(m, &m->rope_cos, static_cast<size_t>(c.max_seq) * (hd / 2));
  rc = rc ? rc : dalloc(m, &m->rope_sin, static_cast<size_t>(c.max_seq) * (hd / 2));
  rc = rc ? rc : dalloc(m, &m->kc, static_cast<size_t>(c.n_layers) * c.max_seq * m->kvd);
  rc = rc ? rc : dalloc(m, &m->vc, static_cast<size_t>(c.n_layers) * c.max_seq * m->kvd);
  rc = rc ? rc : dalloc(m, &m->x, T * c.dim);
  rc = rc ? rc : dalloc(m, &m->qkv, T * m->qkv_w);
  rc = rc ? rc : dalloc(m, &m->attn, T * m->qd);
  rc = rc ? rc : dalloc(m, &m->gu, T * 2 * c.ffn_dim);
  rc = rc ? rc : dalloc(m, &m->logits, T * c.vocab);
  rc = rc ? rc : dalloc(m, &m->d_tokens, T);
  rc = rc ? rc : dalloc(m, &m->d_gen, T + 1);
  rc = rc ? rc : dalloc(m, &m->d_pos, 1);
  rc = rc ? rc : dalloc(m, &m->tickets, 1);
  const size_t fa_pairs = static_cast<size_t>(c.n_heads) * ((m->max_tokens + kFaQ - 1) / kFaQ);
  if (m->hd == 64 || m->hd == 128) {
    rc = rc ? rc : dalloc(m, &m->fa_part, fa_pairs * 2 * kFaQ * (m->hd + 2));
    rc = rc ? rc : dalloc(m, &m->fa_tickets, fa_pairs);
  }
  rc = rc ? rc : dalloc(m, &m->fa_range, 1);
  rc = rc ? rc : dalloc(m, &m->amax_v, kArgmaxBlocks);
  rc = rc ? rc : dalloc(m, &m->amax_i, kArgmaxBlocks);
  if (rc != MRI_OK) {
    mri_llama_free(m);
    return rc;
  }
  // Reserve the context scratch for the largest projection input now: the
  // captured decode graph keeps the scratch address it was captured with.
  const size_t kmax = std::max<size_t>(std::max<size_t>(c.dim, c.ffn_dim), m->qd);
  if (int r = mri::ctx_reserve_scratch(m->ctx, mri::int8_scratch_bytes(T, kmax))) {
    mri_llama_free(m);
    return fail(r, "scratch reservation: %s", mri_last_error());
  }
  cudaMemset(m->tickets, 0, sizeof(int));
  if (m->fa_tickets) cudaMemset(m->fa_tickets, 0, fa_pairs * sizeof(int));
  cudaMemset(m->fa_range, 0, sizeof(int));
  cudaMemset(m->kc, 0, static_cast<size_t>(c.n_layers) * c.max_seq * m->kvd * sizeof(float));
  cudaMemset(m->vc, 0, static_cast<size_t>(c.n_layers) * c.max_seq * m->kvd * sizeof(float));
  // Carve the blobs into QuantizedMatrix views, each starting 256-byte
  // aligned (TMA and vector loads need 16-byte aligned rows and scales).
  size_t wo = 0, so = 0;
  auto view = [&](size_t n_out, size_t k_in) {
    mri_qmatrix q{m->ctx->device, m->w_blob + wo, m->s_blob + so, n_out, k_in, false};
    wo += (n_out * k_in + 255) / 256 * 256;
    so += (n_out + 63) / 64 * 64;
    return q;
  };
  for (uint32_t l = 0; l < c.n_layers; ++l) {
    m->wqkv.push_back(view(m->qkv_w, c.dim));
    m->wo.push_back(view(c.dim, m->qd));
    m->wgu.push_back(view(2 * static_cast<size_t>(c.ffn_dim), c.dim));
    m->wdown.push_back(view(c.dim, c.ffn_dim));
  }
  m->wout = view(c.vocab, c.dim);
  m->fused_decode = mri::matmul_int8_epilogue_supported(m->ctx, 1, &m->wqkv[0]) &&
                    mri::matmul_int8_epilogue_supported(m->ctx, 1, &m->wgu[0]) &&
                    mri::matmul_int8_epilogue_supported(m->ctx, 1, &m->wdown[0]);
  *out = m;
  return MRI_OK;
}

int mri_llama_free(mri_llama* m) {
  if (!m) return MRI_OK;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  if (m->decode_exec) cudaGraphExecDestroy(m->decode_exec);
  for (void* p : m->allocs) cudaFree(p);
  mri_ctx_destroy(m->ctx);
  delete m;
  return MRI_OK;
}

int mri_llama_set_rope(mri_llama* m, const float* cos_t, const float* sin_t) {
  if (!m || !cos_t || !sin_t) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  const size_t n = static_cast<size_t>(m->cfg.max_seq) * (m->hd / 2) * sizeof(float);
  LL_TRY(cudaMemcpy(m->rope_cos, cos_t, n, cudaMemcpyHostToDevice));
  LL_TRY(cudaMemcpy(m->rope_sin, sin_t, n, cudaMemcpyHostToDevice));
  return MRI_OK;
}

int mri_llama_set_embedding(mri_llama* m, const float* token_embd) {
  if (!m || !token_embd) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  LL_TRY(cudaMemcpy(m->embd, token_embd, static_cast<size_t>(m->cfg.vocab) * m->cfg.dim * 4,
                    cudaMemcpyHostToDevice));
  return MRI_OK;
}

int mri_llama_set_norms(mri_llama* m, const float* attn_norm, const float* ffn_norm,
                        const float* output_norm) {
  if (!m || !attn_norm || !ffn_norm || !output_norm) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  const size_t ld = static_cast<size_t>(m->cfg.n_layers) * m->cfg.dim * 4;
  LL_TRY(cudaMemcpy(m->attn_norm, attn_norm, ld, cudaMemcpyHostToDevice));
  LL_TRY(cudaMemcpy(m->ffn_norm, ffn_norm, ld, cudaMemcpyHostToDevice));
  LL_TRY(cudaMemcpy(m->out_norm, output_norm, m->cfg.dim * 4, cudaMemcpyHostToDevice));
  return MRI_OK;
}

static int put_rows(const mri_qmatrix& q, size_t row0, const int8_t* w, const float* s, size_t rows) {
  LL_TRY(cudaMemcpy(q.data + row0 * q.k_in, w, rows * q.k_in, cudaMemcpyHostToDevice));
  LL_TRY(cudaMemcpy(q.scales + row0, s, rows * 4, cudaMemcpyHostToDevice));
  return MRI_OK;
}

int mri_llama_set_layer(mri_llama* m, uint32_t layer, const int8_t* wq, const float* sq,
                        const int8_t* wk, const float* sk, const int8_t* wv, const float* sv,
                        const int8_t* wo, const float* so, const int8_t* wgate, const float* sgate,
                        const int8_t* wup, const float* sup, const int8_t* wdown, const float* sdown) {
  if (!m) return fail(MRI_ERR_INVALID_ARGUMENT, "null model");
  if (layer >= m->cfg.n_layers) return fail(MRI_ERR_INVALID_SHAPE, "layer %u out of range", layer);
  const auto& c = m->cfg;
  if (int rc = put_rows(m->wqkv[layer], 0, wq, sq, m->qd)) return rc;
  if (int rc = put_rows(m->wqkv[layer], m->qd, wk, sk, m->kvd)) return rc;
  if (int rc = put_rows(m->wqkv[layer], m->qd + m->kvd, wv, sv, m->kvd)) return rc;
  if (int rc = put_rows(m->wo[layer], 0, wo, so, c.dim)) return rc;
  {
    // gate and up rows interleaved: row 2i = gate i, row 2i+1 = up i.
    const size_t F = c.ffn_dim, D = c.dim;
    std::vector<int8_t> w(2 * F * D);
    std::vector<float> sc(2 * F);
    for (size_t i = 0; i < F; ++i) {
      std::memcpy(w.data() + (2 * i) * D, wgate + i * D, D);
      std::memcpy(w.data() + (2 * i + 1) * D, wup + i * D, D);
      sc[2 * i] = sgate[i];
      sc[2 * i + 1] = sup[i];
    }
    if (int rc = put_rows(m->wgu[layer], 0, w.data(), sc.data(), 2 * F)) return rc;
  }
  if (int rc = put_rows(m->wdown[layer], 0, wdown, sdown, c.dim)) return rc;
  return MRI_OK;
}

int mri_llama_set_output(mri_llama* m, const int8_t* w, const float* s) {
  if (!m) return fail(MRI_ERR_INVALID_ARGUMENT, "null model");
  return put_rows(m->wout, 0, w, s, m->cfg.vocab);
}

int mri_llama_load_tensor(mri_llama* m, int role, uint32_t layer, int ggml_type,
                          const uint8_t* bytes, size_t len, size_t rows, size_t cols) {
  if (!m) return fail(MRI_ERR_INVALID_ARGUMENT, "null model");
  const auto& c = m->cfg;
  const bool global = role == MRI_TENSOR_TOKEN_EMBD || role == MRI_TENSOR_OUTPUT_NORM ||
                      role == MRI_TENSOR_OUTPUT;
  if (!global && layer >= c.n_layers) return fail(MRI_ERR_INVALID_SHAPE, "layer %u out of range", layer);
  const size_t D = c.dim, F = c.ffn_dim, V = c.vocab, QD = m->qd, KVD = m->kvd;
  // Expected [rows, cols] and destination of each role (the fused Q/K/V and
  // gate/up layouts of mri_llama_set_layer).
  size_t er = 0, ec = D;
  mri::GgufDst d;
  switch (role) {
    case MRI_TENSOR_TOKEN_EMBD: er = V; d.f32 = m->embd; break;
    case MRI_TENSOR_OUTPUT_NORM: er = 1; d.f32 = m->out_norm; break;
    case MRI_TENSOR_ATTN_NORM: er = 1; d.f32 = m->attn_norm + layer * D; break;
    case MRI_TENSOR_FFN_NORM: er = 1; d.f32 = m->ffn_norm + layer * D; break;
    case MRI_TENSOR_OUTPUT:
      er = V;
      d.q = m->wout.data;
      d.scales = m->wout.scales;
      break;
    case MRI_TENSOR_ATTN_Q:
    case MRI_TENSOR_ATTN_K:
    case MRI_TENSOR_ATTN_V: {
      const size_t row0 = role == MRI_TENSOR_ATTN_Q ? 0 : role == MRI_TENSOR_ATTN_K ? QD : QD + KVD;
      er = role == MRI_TENSOR_ATTN_Q ? QD : KVD;
      d.q = m->wqkv[layer].data + row0 * D;
      d.scales = m->wqkv[layer].scales + row0;
      break;
    }
    case MRI_TENSOR_ATTN_OUTPUT:
      er = D;
      ec = QD;
      d.q = m->wo[layer].data;
      d.scales = m->wo[layer].scales;
      break;
    case MRI_TENSOR_FFN_GATE:
    case MRI_TENSOR_FFN_UP: {
      // Row 2i = gate i, row 2i+1 = up i.
      const size_t odd = role == MRI_TENSOR_FFN_UP ? 1 : 0;
      er = F;
      d.q = m->wgu[layer].data + odd * D;
      d.q_stride = 2 * D;
      d.scales = m->wgu[layer].scales + odd;
      d.s_stride = 2;
      break;
    }
    case MRI_TENSOR_FFN_DOWN:
      er = D;
      ec = F;
      d.q = m->wdown[layer].data;
      d.scales = m->wdown[layer].scales;
      break;
    default: return fail(MRI_ERR_INVALID_ARGUMENT, "unknown tensor role %d", role);
  }
  if (rows != er || cols != ec)
    return fail(MRI_ERR_SHAPE_MISMATCH, "tensor role %d: expected [%zu, %zu], got [%zu, %zu]", role,
                er, ec, rows, cols);
  if (d.q && !d.q_stride) d.q_stride = ec;
  LL_TRY(cudaSetDevice(m->ctx->device));
  std::string err;
  if (int rc = mri::gguf_to_device(m->ctx->stream, ggml_type, bytes, len, rows, cols, d, &err))
    return fail(rc, "%s", err.c_str());
  return MRI_OK;
}

int mri_llama_init_random(mri_llama* m, uint64_t seed) {
  if (!m) return fail(MRI_ERR_INVALID_ARGUMENT, "null model");
  const auto& c = m->cfg;
  const BlobLayout b = blob_layout(m);
  const int sms = m->ctx->dev.sm_count;
  cudaStream_t st = m->ctx->stream;
  fill_i8_kernel<<<sms * 8, 256, 0, st>>>(m->w_blob, b.total_w, seed);
  // Per-channel scales of N(0, 0.02)-like weights quantized to int8.
  fill_f32_kernel<<<sms * 8, 256, 0, st>>>(m->s_blob, b.total_s, seed + 1, 4e-4f, 8e-4f);
  fill_f32_kernel<<<sms * 8, 256, 0, st>>>(m->embd, static_cast<size_t>(c.vocab) * c.dim, seed + 2,
                                           -1.0f, 1.0f);
  fill_f32_kernel<<<sms, 256, 0, st>>>(m->attn_norm, static_cast<size_t>(c.n_layers) * c.dim, seed + 3,
                                       1.0f, 1.0f);
  fill_f32_kernel<<<sms, 256, 0, st>>>(m->ffn_norm, static_cast<size_t>(c.n_layers) * c.dim, seed + 4,
                                       1.0f, 1.0f);
  fill_f32_kernel<<<1, 256, 0, st>>>(m->out_norm, c.dim, seed + 5, 1.0f, 1.0f);
  LL_TRY(cudaGetLastError());
  LL_TRY(cudaStreamSynchronize(st));
  return MRI_OK;
}

int mri_llama_forward(mri_llama* m, const uint32_t* tokens, size_t n, float* logits) {
  if (!m || !tokens) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  g_model_error.clear();
  if (int rc = check_tokens(m, tokens, n)) return rc;
  cudaSetDevice(m->ctx->device);
  return forward_rows(m, tokens, n, 0, logits);
}

int mri_llama_forward_at(mri_llama* m, const uint32_t* tokens, size_t n, size_t start_pos,
                         float* logits) {
  if (!m || !tokens) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  g_model_error.clear();
  if (int rc = check_tokens(m, tokens, n)) return rc;
  if (start_pos > m->cfg.max_seq || n > m->cfg.max_seq - start_pos)
    return fail(MRI_ERR_INVALID_SHAPE, "forward_at: positions [%zu, %zu) exceed max_seq %u", start_pos,
                start_pos + n, m->cfg.max_seq);
  cudaSetDevice(m->ctx->device);
  return forward_rows(m, tokens, n, start_pos, logits);
}

int mri_llama_block_forward(mri_llama* m, uint32_t layer, const float* x, size_t n, size_t start_pos,
                            float* out) {
  if (!m || !x || !out) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  g_model_error.clear();
  if (layer >= m->cfg.n_layers)
    return fail(MRI_ERR_INVALID_SHAPE, "layer %u >= n_layers %u", layer, m->cfg.n_layers);
  if (n == 0) return fail(MRI_ERR_INVALID_SHAPE, "block forward: input must have at least one row");
  if (start_pos > m->cfg.max_seq || n > m->cfg.max_seq - start_pos)
    return fail(MRI_ERR_INVALID_SHAPE, "block forward: positions [%zu, %zu) exceed max_seq %u", start_pos,
                start_pos + n, m->cfg.max_seq);
  cudaSetDevice(m->ctx->device);
  cudaStream_t st = m->ctx->stream;
  const size_t bytes = n * m->cfg.dim * sizeof(float);
  for (int attempt = 0;; ++attempt) {
    LL_TRY(cudaMemcpyAsync(m->x, x, bytes, cudaMemcpyHostToDevice, st));
    if (int rc = run_blocks(m, n, static_cast<int>(start_pos), false, layer, layer + 1)) return rc;
    LL_TRY(cudaMemcpyAsync(out, m->x, bytes, cudaMemcpyDeviceToHost, st));
    LL_TRY(cudaStreamSynchronize(st));
    const bool redo = attempt == 0 && take_range_flag(m);
    m->cuda_core_attn = redo;
    if (!redo) break;
    m->attn_fallbacks++;
  }
  return mri_ctx_check_device_status(m->ctx) ? fail(MRI_ERR_TIMEOUT, "%s", mri_last_error()) : MRI_OK;
}

int mri_llama_set_option(mri_llama* m, int option, int value) {
  if (!m) return fail(MRI_ERR_INVALID_ARGUMENT, "null model");
  if (int rc = mri_ctx_set_option(m->ctx, option, value)) return fail(rc, "%s", mri_last_error());
  return MRI_OK;
}

int mri_llama_attention_fallbacks(const mri_llama* m, size_t* count) {
  if (!m || !count) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  *count = m->attn_fallbacks;
  return MRI_OK;
}

int mri_llama_forward_decode(mri_llama* m, uint32_t token, size_t pos, float* logits) {
  if (!m) return fail(MRI_ERR_INVALID_ARGUMENT, "null model");
  g_model_error.clear();
  if (token >= m->cfg.vocab)
    return fail(MRI_ERR_INVALID_SHAPE, "token id %u >= vocab_size %u", token, m->cfg.vocab);
  if (pos >= m->cfg.max_seq)
    return fail(MRI_ERR_INVALID_SHAPE, "position %zu beyond max_seq %u", pos, m->cfg.max_seq);
  cudaSetDevice(m->ctx->device);
  if (int rc = ensure_decode_graph(m)) return rc;
  cudaStream_t st = m->ctx->stream;
  const int p = static_cast<int>(pos);
  LL_TRY(cudaMemcpyAsync(m->d_tokens, &token, sizeof(uint32_t), cudaMemcpyHostToDevice, st));
  LL_TRY(cudaMemcpyAsync(m->d_pos, &p, sizeof(int), cudaMemcpyHostToDevice, st));
  LL_TRY(cudaGraphLaunch(m->decode_exec, st));
  if (logits)
    LL_TRY(cudaMemcpyAsync(logits, m->logits, m->cfg.vocab * 4, cudaMemcpyDeviceToHost, st));
  LL_TRY(cudaStreamSynchronize(st));
  return mri_ctx_check_device_status(m->ctx) ? fail(MRI_ERR_TIMEOUT, "%s", mri_last_error()) : MRI_OK;
}

int mri_llama_generate_greedy(mri_llama* m, const uint32_t* prompt, size_t n_prompt,
                              size_t n_decode, uint32_t* out_tokens, float* prefill_ms,
                              float* decode_ms) {
  if (!m || !prompt) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  g_model_error.clear();
  if (int rc = check_tokens(m, prompt, n_prompt)) return rc;
  if (n_prompt + n_decode > m->cfg.max_seq)
    return fail(MRI_ERR_INVALID_SHAPE, "prompt %zu + %zu decode steps exceed max_seq %u", n_prompt,
                n_decode, m->cfg.max_seq);
  cudaSetDevice(m->ctx->device);
  if (int rc = ensure_decode_graph(m)) return rc;
  cudaStream_t st = m->ctx->stream;
  cudaEvent_t e0, e1, e2;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventCreate(&e2);
  int rc = MRI_OK;
  for (int attempt = 0;; ++attempt) {
    cudaEventRecord(e0, st);
    rc = prefill(m, prompt, n_prompt);
    if (rc == MRI_OK) rc = lm_head(m, n_prompt - 1, 1);
    if (rc == MRI_OK) {
      const int p = static_cast<int>(n_prompt) - 1;  // argmax advances it to n_prompt
      cudaMemcpyAsync(m->d_pos, &p, sizeof(int), cudaMemcpyHostToDevice, st);
      rc = launch_argmax(m);
      cudaEventRecord(e1, st);
      for (size_t i = 0; i < n_decode && rc == MRI_OK; ++i)
        if (cudaGraphLaunch(m->decode_exec, st) != cudaSuccess) rc = fail(MRI_ERR_CUDA, "graph launch");
      cudaEventRecord(e2, st);
      if (out_tokens)
        cudaMemcpyAsync(out_tokens, m->d_gen + n_prompt, (n_decode + 1) * sizeof(uint32_t),
                        cudaMemcpyDeviceToHost, st);
    }
    cudaError_t e = cudaStreamSynchronize(st);
    if (rc == MRI_OK && e != cudaSuccess) rc = fail(MRI_ERR_CUDA, "%s", cudaGetErrorString(e));
    // A prompt whose q, k or v left the f16 range: the whole call again, the
    // prefill attention on the f32 kernel.
    const bool redo = rc == MRI_OK && attempt == 0 && take_range_flag(m);
    m->cuda_core_attn = redo;
    if (!redo) break;
    m->attn_fallbacks++;
  }
  if (rc == MRI_OK) {
    float a = 0, b = 0;
    cudaEventElapsedTime(&a, e0, e1);
    cudaEventElapsedTime(&b, e1, e2);
    if (prefill_ms) *prefill_ms = a;
    if (decode_ms) *decode_ms = b;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaEventDestroy(e2);
  if (rc == MRI_OK && mri_ctx_check_device_status(m->ctx))
    rc = fail(MRI_ERR_TIMEOUT, "%s", mri_last_error());
  return rc;
}

int mri_llama_launches_per_decode_step(const mri_llama* m, size_t* count) {
  if (!m || !count) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  *count = m->graph_kernels;  // kernel nodes of the captured decode step (0 before capture)
  return MRI_OK;
}

}  // extern "C"
