// abi.cu — the C ABI (include/mri_gpu.h): contexts, device-resident weight
// handles, argument validation with the reference's error classes, and
// dispatch to the kernels.  No CPU compute path exists here: every product
// runs on the GPU or the call fails.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "internal.h"
#include "mri_gpu.h"

using mri::ActArgs;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(MRI_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

#define MRI_CUDA_TRY(expr)                                   \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return cuda_fail(_e, #expr);      \
  } while (0)

// Device allocations of weights carry this many bytes of zeroed slack: bulk
// copies round their size up to 16 bytes and may read past the last row.
constexpr size_t kWeightPad = 256;

int use_device(int device) {
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (cur != device) MRI_CUDA_TRY(cudaSetDevice(device));
  return MRI_OK;
}

int enter(mri_ctx* ctx) {
  if (!ctx) return fail(MRI_ERR_INVALID_ARGUMENT, "null context");
  g_last_error.clear();
  return use_device(ctx->device);
}

int check_k(const char* fn, size_t m, size_t k, size_t k_w);

// Scratch is one growing device buffer per context, carved by the callers.
int ensure_scratch(mri_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->scratch_bytes) return MRI_OK;
  if (ctx->scratch) {
    MRI_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    MRI_CUDA_TRY(cudaFree(ctx->scratch));
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
  }
  const size_t sz = std::max<size_t>(bytes, 1 << 20);
  MRI_CUDA_TRY(cudaMalloc(&ctx->scratch, sz));
  ctx->scratch_bytes = sz;
  return MRI_OK;
}

size_t al(size_t v) { return (v + 255) / 256 * 256; }

// Bytes of the quantizer's maxima area at the front of scratch.
size_t amax_bytes(size_t m) { return al(2 * std::max(m, mri::kQuantPartials) * sizeof(float)); }

template <typename T>
int upload_bytes(const T* host, size_t count, T** dev) {
  const size_t bytes = count * sizeof(T);
  void* p = nullptr;
  MRI_CUDA_TRY(cudaMalloc(&p, bytes + kWeightPad));
  cudaError_t e = cudaMemset(p, 0, bytes + kWeightPad);
  if (e == cudaSuccess && bytes) e = cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "weight upload");
  }
  *dev = static_cast<T*>(p);
  return MRI_OK;
}

}  // namespace

namespace mri {
int ctx_reserve_scratch(::mri_ctx* ctx, size_t bytes) { return ensure_scratch(ctx, bytes); }
size_t int8_scratch_bytes(size_t m, size_t k) {
  return amax_bytes(m) + al(m * sizeof(float)) + al(m * k);
}
}  // namespace mri

namespace {

// ── INT8 dispatch ────────────────────────────────────────────────────────────
// `act` describes the full [m, K] activation set.  Small m uses the fused
// streaming GEMV; larger m quantizes once (per-tensor scale over all rows,
// as the reference does) and runs the tensor-core GEMM or, where that does
// not apply, the GEMV over 8-row chunks.
bool stream_gemv_applies(const mri_ctx* ctx, size_t m, const mri_qmatrix* w) {
  return m >= 1 && m <= 8 && (reinterpret_cast<uintptr_t>(w->data) & 15) == 0 &&
         mri::gemv_i8_tma_supported(ctx->dev, static_cast<int>(m), w->k_in);
}

int run_int8(mri_ctx* ctx, ActArgs act, const mri_qmatrix* w, size_t m, float* out,
             int32_t* acc, const float* residual = nullptr, const mri::EpiArgs* epi = nullptr) {
  const size_t N = w->n_out, K = w->k_in;
  if (m == 0 || N == 0) return MRI_OK;
  cudaStream_t st = ctx->stream;
  const bool f32_in = act.mode == mri::ACT_F32_PER_TENSOR || act.mode == mri::ACT_F32_PER_ROW;

  const bool w_aligned = (reinterpret_cast<uintptr_t>(w->data) & 15) == 0;
  if (stream_gemv_applies(ctx, m, w)) {
    // An f32 input too long for the register prologue (M*K > 12288) would be
    // read twice from L2 by every CTA; quantize it once instead (two small
    // kernels the GEMV's weight prefetch overlaps) and stream int8 rows.
    if (f32_in && !epi && mri::reg_vec(static_cast<int>(m), K, &act) == 0) {
      const size_t need = amax_bytes(m) + al(m * sizeof(float)) + al(m * K);
      if (int rc = ensure_scratch(ctx, need)) return rc;
      float* amax = reinterpret_cast<float*>(ctx->scratch);
      float* scales = reinterpret_cast<float*>(ctx->scratch + amax_bytes(m));
      int8_t* q = reinterpret_cast<int8_t*>(ctx->scratch + amax_bytes(m) + al(m * sizeof(float)));
      const int per_row = act.mode == mri::ACT_F32_PER_ROW;
      MRI_CUDA_TRY(mri::launch_quantize(ctx->dev, st, act.x, m, K, per_row, q, scales, amax, &ctx->ls,
                                        act.norm_w, act.eps, act.swiglu, ctx->d_sync, ctx->d_status));
      ActArgs a;
      a.xq = q;
      a.mode = per_row ? mri::ACT_I8_DEV_ROW_SCALE : mri::ACT_I8_DEV_SCALE;
      a.scale_dev = scales;
      MRI_CUDA_TRY(mri::launch_gemv_i8_tma(ctx->dev, st, static_cast<int>(m), w->data, w->scales, N,
                                           K, a, out, acc, ctx->d_status, &ctx->ls, residual));
      return MRI_OK;
    }
    MRI_CUDA_TRY(mri::launch_gemv_i8_tma(ctx->dev, st, static_cast<int>(m), w->data, w->scales, N,
                                         K, act, out, acc, ctx->d_status, &ctx->ls, residual, epi));
    return MRI_OK;
  }
  if (epi) return fail(MRI_ERR_INVALID_ARGUMENT, "pair epilogue needs the streaming GEMV path (m <= 8, K %% 16 == 0)");

  // Materialize quantized activations (and device scales) if needed.
  const int8_t* xq = act.xq;
  const float* sdev = act.scale_dev;
  int per_row = act.mode == mri::ACT_I8_DEV_ROW_SCALE || act.mode == mri::ACT_F32_PER_ROW;
  if (f32_in || act.mode == mri::ACT_I8_HOST_SCALE) {
    const size_t need = amax_bytes(m) + al(m * sizeof(float)) + al(m * K);
    if (int rc = ensure_scratch(ctx, need)) return rc;
    float* amax = reinterpret_cast<float*>(ctx->scratch);
    float* scales = reinterpret_cast<float*>(ctx->scratch + amax_bytes(m));
    int8_t* q = reinterpret_cast<int8_t*>(ctx->scratch + amax_bytes(m) + al(m * sizeof(float)));
    if (f32_in) {
      MRI_CUDA_TRY(mri::launch_quantize(ctx->dev, st, act.x, m, K, per_row, q, scales, amax,
                                        &ctx->ls, act.norm_w, act.eps, act.swiglu, ctx->d_sync,
                                        ctx->d_status));
      xq = q;
    } else {
      MRI_CUDA_TRY(cudaMemcpyAsync(scales, &act.scale_host, sizeof(float),
                                   cudaMemcpyHostToDevice, st));
      per_row = 0;
    }
    sdev = scales;
  }

  if (w_aligned && mri::gemm_i8_tc_supported(ctx->dev, m, N, K) &&
      (reinterpret_cast<uintptr_t>(xq) & 15) == 0) {
    MRI_CUDA_TRY(mri::launch_gemm_i8_tc(ctx->dev, st, xq, sdev, per_row, w->data, w->scales, m, N,
                                        K, out, acc, ctx->d_status, &ctx->ls, residual));
    return MRI_OK;
  }
  for (size_t m0 = 0; m0 < m; m0 += 8) {
    const int mc = static_cast<int>(std::min<size_t>(8, m - m0));
    ActArgs a;
    a.xq = xq + m0 * K;
    a.mode = per_row ? mri::ACT_I8_DEV_ROW_SCALE : mri::ACT_I8_DEV_SCALE;
    a.scale_dev = per_row ? sdev + m0 : sdev;
    float* o = out + m0 * N;
    int32_t* ac = acc ? acc + m0 * N : nullptr;
    if (w_aligned && mri::gemv_i8_tma_supported(ctx->dev, mc, K)) {
      MRI_CUDA_TRY(mri::launch_gemv_i8_tma(ctx->dev, st, mc, w->data, w->scales, N, K, a, o, ac,
                                           ctx->d_status, &ctx->ls));
    } else {
      MRI_CUDA_TRY(mri::launch_gemv_i8_generic(ctx->dev, st, mc, w->data, w->scales, N, K, a, o,
                                               ac, &ctx->ls));
    }
  }
  if (residual) MRI_CUDA_TRY(mri::launch_add_residual(ctx->dev, st, out, residual, m * N, &ctx->ls));
  return MRI_OK;
}

}  // namespace

int mri::set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int mri::quantize_to_scratch(::mri_ctx* ctx, const float* x, size_t m, size_t k, int8_t** q,
                             float** scale_dev) {
  if (int rc = enter(ctx)) return rc;
  const size_t need = amax_bytes(m) + al(sizeof(float)) + al(m * k);
  if (int rc = ensure_scratch(ctx, need)) return rc;
  float* amax = reinterpret_cast<float*>(ctx->scratch);
  *scale_dev = reinterpret_cast<float*>(ctx->scratch + amax_bytes(m));
  *q = reinterpret_cast<int8_t*>(ctx->scratch + amax_bytes(m) + al(sizeof(float)));
  MRI_CUDA_TRY(mri::launch_quantize(ctx->dev, ctx->stream, x, m, k, 0, *q, *scale_dev, amax, &ctx->ls,
                                    nullptr, 0.0f, 0, ctx->d_sync, ctx->d_status));
  return MRI_OK;
}

int mri::matmul_int8_act(::mri_ctx* ctx, const ActArgs& act, const ::mri_qmatrix* w, size_t m,
                         float* out) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  return run_int8(ctx, act, w, m, out, nullptr);
}

bool mri::stream_gemv_ok(const ::mri_ctx* ctx, size_t m, const ::mri_qmatrix* w) {
  return ctx && w && stream_gemv_applies(ctx, m, w);
}

int mri::matmul_int8_gather(::mri_ctx* ctx, const float* x, size_t m, size_t k,
                            const ::mri_qmatrix* w, const EpiArgs& e) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (int rc = check_k("sharded matmul", m, k, w->k_in)) return rc;
  if (!stream_gemv_applies(ctx, m, w))
    return fail(MRI_ERR_INVALID_ARGUMENT, "peer gather needs the streaming GEMV (m <= 8, K %% 16 == 0)");
  ActArgs a;
  a.x = x;
  a.mode = mri::ACT_F32_PER_TENSOR;
  MRI_CUDA_TRY(mri::launch_gemv_i8_tma(ctx->dev, ctx->stream, static_cast<int>(m), w->data, w->scales,
                                       w->n_out, w->k_in, a, e.g_out, nullptr, ctx->d_status, &ctx->ls,
                                       nullptr, &e));
  MRI_CUDA_TRY(mri::launch_gather_collect(ctx->dev, ctx->stream, e, static_cast<int>(m), ctx->d_status,
                                          &ctx->ls));
  return MRI_OK;
}

bool mri::matmul_int8_epilogue_supported(const ::mri_ctx* ctx, size_t m, const ::mri_qmatrix* w) {
  return ctx && w && m == 1 && w->n_out % 2 == 0 && stream_gemv_applies(ctx, m, w);
}

int mri::matmul_int8_fused(::mri_ctx* ctx, const float* x, size_t m, size_t k, const float* norm_w,
                           float eps, int swiglu, const ::mri_qmatrix* w, const float* residual,
                           float* out, const EpiArgs* epi, int pre_stages) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (int rc = check_k("matmul_int8_fused", m, k, w->k_in)) return rc;
  ActArgs a;
  a.x = x;
  a.mode = mri::ACT_F32_PER_TENSOR;
  a.norm_w = norm_w;
  a.eps = eps;
  a.swiglu = swiglu;
  a.pre_stages = pre_stages;
  if (epi && (residual || w->n_out % 2 || m != 1))
    return fail(MRI_ERR_INVALID_ARGUMENT, "pair epilogue needs one row, even N and no residual");
  return run_int8(ctx, a, w, m, out, nullptr, residual, epi);
}

namespace {

// Chunks of at most 8 activation rows.  The streaming kernel quantizes its
// rows per row in its prologue (q8_direct.rs:264); the MMA kernel (2..8 rows)
// and the generic one read activations quantized per row once for the whole
// call (measured: the quantizer kernel in front of the MMA kernel costs less
// than the same reductions in its prologue).
int run_q8_0(mri_ctx* ctx, const float* x, size_t m, const mri_q8_0_matrix* w, float* out) {
  const size_t N = w->n_out, K = w->k_in;
  if (m == 0 || N == 0) return MRI_OK;
  cudaStream_t st = ctx->stream;
  int8_t* q = nullptr;
  float* scales = nullptr;
  for (size_t m0 = 0; m0 < m; m0 += 8) {
    const int mc = static_cast<int>(std::min<size_t>(8, m - m0));
    const bool pin = mri::q8_0_mma_supported(ctx->dev, mc, K);
    if (!pin && K > 0 && mri::gemv_q8_0_tma_supported(ctx->dev, mc, K)) {
      MRI_CUDA_TRY(mri::launch_gemv_q8_0_tma(ctx->dev, st, mc, w->data, N, K, x + m0 * K,
                                             out + m0 * N, ctx->d_status, &ctx->ls));
      continue;
    }
    if (q == nullptr) {
      const size_t need = amax_bytes(m) + al(m * sizeof(float)) + al(m * K);
      if (int rc = ensure_scratch(ctx, need)) return rc;
      float* amax = reinterpret_cast<float*>(ctx->scratch);
      scales = reinterpret_cast<float*>(ctx->scratch + amax_bytes(m));
      q = reinterpret_cast<int8_t*>(ctx->scratch + amax_bytes(m) + al(m * sizeof(float)));
      MRI_CUDA_TRY(mri::launch_quantize(ctx->dev, st, x, m, K, 1, q, scales, amax, &ctx->ls));
    }
    if (pin) {
      mri::ActArgs a;
      a.xq = q + m0 * K;
      a.scale_dev = scales + m0;
      a.mode = mri::ACT_I8_DEV_ROW_SCALE;
      MRI_CUDA_TRY(mri::launch_gemv_q8_0_mma(ctx->dev, st, mc, w->data, N, K, a, out + m0 * N,
                                             ctx->d_status, &ctx->ls));
    } else {
      MRI_CUDA_TRY(mri::launch_gemv_q8_0_generic(ctx->dev, st, mc, w->data, N, K, q + m0 * K,
                                                 scales + m0, out + m0 * N, &ctx->ls));
    }
  }
  return MRI_OK;
}

int run_q4_0(mri_ctx* ctx, const float* x, size_t m, const mri_q4_0_matrix* w, float* out) {
  const size_t N = w->n_out, K = w->k;
  if (m == 0 || N == 0) return MRI_OK;
  cudaStream_t st = ctx->stream;
  const bool tma = K > 0 && mri::gemv_q4_0_tma_supported(ctx->dev, static_cast<int>(std::min<size_t>(m, 8)), K);
  const bool x_vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  uint32_t* xs = nullptr;  // split activations of all m rows, made on first use
  for (size_t m0 = 0; m0 < m; m0 += 8) {
    const int mc = static_cast<int>(std::min<size_t>(8, m - m0));
    if (mc == 1 && mri::gemv_q4_0_limb_supported(ctx->dev, K, x + m0 * K)) {
      MRI_CUDA_TRY(mri::launch_gemv_q4_0_limb(ctx->dev, st, w->data, N, K, x + m0 * K, out + m0 * N,
                                              ctx->d_status, &ctx->ls));
    } else if (x_vec && mri::q4_0_mma_supported(ctx->dev, mc, K)) {
      if (xs == nullptr) {
        if (int rc = ensure_scratch(ctx, al(mri::q4_0_split_bytes(m, K)))) return rc;
        xs = reinterpret_cast<uint32_t*>(ctx->scratch);
        MRI_CUDA_TRY(mri::launch_q4_0_split(ctx->dev, st, x, m, K, xs, &ctx->ls));
      }
      MRI_CUDA_TRY(mri::launch_gemv_q4_0_mma(
          ctx->dev, st, mc, w->data, N, K,
          reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(xs) + mri::q4_0_split_bytes(m0, K)),
          out + m0 * N, ctx->d_status, &ctx->ls));
    } else if (tma) {
      MRI_CUDA_TRY(mri::launch_gemv_q4_0_tma(ctx->dev, st, mc, w->data, N, K, x + m0 * K,
                                             out + m0 * N, ctx->d_status, &ctx->ls));
    } else {
      MRI_CUDA_TRY(mri::launch_gemv_q4_0_generic(ctx->dev, st, mc, w->data, N, K, x + m0 * K,
                                                 out + m0 * N, &ctx->ls));
    }
  }
  return MRI_OK;
}

int check_act_len(const char* fn, size_t act_len, size_t m, size_t k) {
  // int8.rs:68-78 / parallel.rs:315-325
  if (act_len != m * k)
    return fail(MRI_ERR_INVALID_SHAPE, "%s: act_q.len()=%zu != m*k=%zu*%zu=%zu", fn, act_len, m, k,
                m * k);
  return MRI_OK;
}

int check_k(const char* fn, size_t m, size_t k, size_t k_w) {
  // int8.rs:127-132, q8_direct.rs:241-246, q4_0.rs:114-119
  if (k != k_w)
    return fail(MRI_ERR_SHAPE_MISMATCH, "%s: ShapeMismatch expected [%zu, %zu], got [%zu, %zu]", fn,
                m, k_w, m, k);
  return MRI_OK;
}

// Reads and clears the mapped status word (the stream must be idle).  After a
// timeout the quantizer's grid-barrier words may hold a partial count; they
// are cleared too.
int read_status(mri_ctx* ctx) {
  volatile int* hs = ctx->h_status;
  const int st = *hs;
  if (st != MRI_OK) {
    *hs = MRI_OK;
    if (ctx->d_sync) cudaMemset(ctx->d_sync, 0, 2 * sizeof(unsigned));
    return fail(st, "a device-side bounded wait timed out");
  }
  return MRI_OK;
}

// Host-call staging: [x | act_q] [out] [acc] in scratch after the quantizer area.
struct HostStage {
  uint8_t* in;
  float* out;
  int32_t* acc;
};

int host_stage(mri_ctx* ctx, size_t in_bytes, size_t out_bytes, size_t acc_bytes, size_t quant_m,
               size_t quant_k, HostStage* hs) {
  const size_t quant = amax_bytes(quant_m) + al(quant_m * sizeof(float)) + al(quant_m * quant_k);
  const size_t need = quant + al(in_bytes) + al(out_bytes) + al(acc_bytes);
  if (int rc = ensure_scratch(ctx, need)) return rc;
  hs->in = ctx->scratch + quant;
  hs->out = reinterpret_cast<float*>(hs->in + al(in_bytes));
  hs->acc = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(hs->out) + al(out_bytes));
  return MRI_OK;
}

// The device mapping of a caller's host buffer when it is page-locked and
// mapped into the device's address space (e.g. from cudaHostAlloc), else null.
float* mapped_host(void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a.type != cudaMemoryTypeHost || a.devicePointer == nullptr) return nullptr;
  return static_cast<float*>(a.devicePointer);
}

// A host call's f32 result (n floats staged at `dev`) into the caller's
// buffer: into a pinned buffer by a copy kernel writing its device mapping
// (launched behind the product, no copy-engine round trip), else by a copy.
int copy_result(mri_ctx* ctx, float* out, const float* dev, size_t n) {
  if (n == 0) return MRI_OK;
  float* mapped = n % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 ? mapped_host(out) : nullptr;
  if (mapped) {
    const cudaError_t e = mri::launch_copy_out(ctx->dev, ctx->stream, dev, mapped, n, &ctx->ls);
    return e == cudaSuccess ? MRI_OK : cuda_fail(e, "copy_out");
  }
  MRI_CUDA_TRY(cudaMemcpyAsync(out, dev, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
  return MRI_OK;
}

// The quantizer area at the front of scratch must not overlap the host
// staging area, so host calls reserve it explicitly (host_stage quant_*),
// and run_int8/run_q8_0 carve from offset 0 within that reservation.

}  // namespace

extern "C" {

int mri_abi_version(void) { return MRI_ABI_VERSION; }

const char* mri_last_error(void) { return g_last_error.c_str(); }

static int ctx_create(int device, void* stream, bool own, mri_ctx** out) {
  if (!out) return fail(MRI_ERR_INVALID_ARGUMENT, "null output pointer");
  *out = nullptr;
  g_last_error.clear();
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= count)
    return fail(MRI_ERR_CUDA, "device %d not present (%d devices)", device, count);
  MRI_CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  MRI_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(MRI_ERR_CUDA, "device %d is sm_%d%d; this library is built for sm_100a", device,
                prop.major, prop.minor);
  mri_ctx* c = new mri_ctx();
  c->device = device;
  c->dev.device = device;
  c->dev.sm_count = prop.multiProcessorCount;
  c->dev.max_smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
  c->dev.cc_major = prop.major;
  c->dev.cc_minor = prop.minor;
  c->dev.l2_bytes = prop.l2CacheSize;
  if (own) {
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      delete c;
      return cuda_fail(e, "cudaStreamCreate");
    }
  } else {
    c->stream = static_cast<cudaStream_t>(stream);
  }
  c->own_stream = own;
  // The status word lives in mapped pinned host memory: kernels store to it
  // through the device alias and the host reads it after a stream sync, with
  // no extra copy.
  e = cudaHostAlloc(&c->h_status, sizeof(int), cudaHostAllocMapped);
  if (e == cudaSuccess) {
    *c->h_status = 0;
    e = cudaHostGetDevicePointer(&c->d_status, c->h_status, 0);
  }
  if (e == cudaSuccess) e = cudaMalloc(&c->d_sync, 256);
  if (e == cudaSuccess) e = cudaMemset(c->d_sync, 0, 256);
  if (e != cudaSuccess) {
    if (c->d_sync) cudaFree(c->d_sync);
    if (c->h_status) cudaFreeHost(c->h_status);
    if (own) cudaStreamDestroy(c->stream);
    delete c;
    return cuda_fail(e, "status word");
  }
  *out = c;
  return MRI_OK;
}

int mri_ctx_create(int device, mri_ctx** out) { return ctx_create(device, nullptr, true, out); }

int mri_ctx_create_on_stream(int device, void* cuda_stream, mri_ctx** out) {
  return ctx_create(device, cuda_stream, false, out);
}

int mri_ctx_destroy(mri_ctx* ctx) {
  if (!ctx) return MRI_OK;
  use_device(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->h_status) cudaFreeHost(ctx->h_status);
  if (ctx->d_sync) cudaFree(ctx->d_sync);
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return MRI_OK;
}

int mri_ctx_synchronize(mri_ctx* ctx) {
  if (int rc = enter(ctx)) return rc;
  MRI_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return MRI_OK;
}

void* mri_ctx_stream(mri_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int mri_ctx_check_device_status(mri_ctx* ctx) {
  if (int rc = enter(ctx)) return rc;
  MRI_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return read_status(ctx);
}

uint64_t mri_ctx_launch_count(const mri_ctx* ctx) { return ctx ? ctx->ls.launches : 0; }

namespace {
int* option_slot(mri_ctx* ctx, int option) {
  mri::Options& o = ctx->dev.opt;
  switch (option) {
    case MRI_OPT_PDL: return &o.pdl;
    case MRI_OPT_GEMM_BN: return &o.gemm_bn;
    case MRI_OPT_GEMM_2CTA: return &o.gemm_2cta;
    case MRI_OPT_Q8_MMA: return &o.q8_mma;
    case MRI_OPT_Q4_MMA: return &o.q4_mma;
    case MRI_OPT_TC_ATTN: return &o.tc_attn;
    case MRI_OPT_FA_SPLIT: return &o.fa_split;
    case MRI_OPT_SHARD_PEER: return &o.shard_peer;
    case MRI_OPT_GEMM_PAIR: return &o.gemm_pair;
    case MRI_OPT_Q4_LIMB: return &o.q4_limb;
    default: return nullptr;
  }
}
}  // namespace

int mri_ctx_set_option(mri_ctx* ctx, int option, int value) {
  if (!ctx) return fail(MRI_ERR_INVALID_ARGUMENT, "null context");
  int* slot = option_slot(ctx, option);
  if (!slot) return fail(MRI_ERR_INVALID_ARGUMENT, "unknown option %d", option);
  bool ok = true;
  switch (option) {
    case MRI_OPT_GEMM_BN: ok = value == 0 || (value >= 128 && value <= 256 && value % 32 == 0); break;
    case MRI_OPT_FA_SPLIT: ok = value >= 0; break;
    case MRI_OPT_SHARD_PEER: ok = value >= 0 && value <= 2; break;
    case MRI_OPT_GEMM_PAIR: ok = value >= 0 && value <= 2; break;
    default: ok = value == 0 || value == 1;
  }
  if (!ok) return fail(MRI_ERR_INVALID_ARGUMENT, "value %d out of range for option %d", value, option);
  *slot = value;
  return MRI_OK;
}

int mri_ctx_get_option(mri_ctx* ctx, int option, int* value) {
  if (!ctx || !value) return fail(MRI_ERR_INVALID_ARGUMENT, "null context or output");
  const int* slot = option_slot(ctx, option);
  if (!slot) return fail(MRI_ERR_INVALID_ARGUMENT, "unknown option %d", option);
  *value = *slot;
  return MRI_OK;
}

// ── weights ──────────────────────────────────────────────────────────────────

int mri_qmatrix_upload_rows(mri_ctx* ctx, const int8_t* data, const float* scales, size_t n_out,
                            size_t k_in, size_t row_begin, size_t row_end, mri_qmatrix** out) {
  if (int rc = enter(ctx)) return rc;
  if (!out) return fail(MRI_ERR_INVALID_ARGUMENT, "null output pointer");
  if (row_begin > row_end || row_end > n_out)
    return fail(MRI_ERR_INVALID_SHAPE, "row range [%zu, %zu) outside n_out=%zu", row_begin,
                row_end, n_out);
  const size_t rows = row_end - row_begin;
  if ((rows * k_in > 0 && !data) || (rows > 0 && !scales))
    return fail(MRI_ERR_INVALID_ARGUMENT, "null weight pointer");
  mri_qmatrix* w = new mri_qmatrix{ctx->device, nullptr, nullptr, rows, k_in, true};
  int rc = upload_bytes(data ? data + row_begin * k_in : data, rows * k_in, &w->data);
  if (rc == MRI_OK) rc = upload_bytes(scales ? scales + row_begin : scales, rows, &w->scales);
  if (rc != MRI_OK) {
    if (w->data) cudaFree(w->data);
    delete w;
    return rc;
  }
  *out = w;
  return MRI_OK;
}

int mri_qmatrix_upload(mri_ctx* ctx, const int8_t* data, const float* scales, size_t n_out,
                       size_t k_in, mri_qmatrix** out) {
  return mri_qmatrix_upload_rows(ctx, data, scales, n_out, k_in, 0, n_out, out);
}

int mri_qmatrix_free(mri_qmatrix* w) {
  if (!w) return MRI_OK;
  use_device(w->device);
  if (w->owns) {
    cudaFree(w->data);
    cudaFree(w->scales);
  }
  delete w;
  return MRI_OK;
}

int mri_qmatrix_dims(const mri_qmatrix* w, size_t* n_out, size_t* k_in) {
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null matrix");
  if (n_out) *n_out = w->n_out;
  if (k_in) *k_in = w->k_in;
  return MRI_OK;
}

int mri_qmatrix_from_gguf(mri_ctx* ctx, int ggml_type, const uint8_t* bytes, size_t len,
                          size_t n_out, size_t k_in, mri_qmatrix** out) {
  if (int rc = enter(ctx)) return rc;
  if (!out) return fail(MRI_ERR_INVALID_ARGUMENT, "null output pointer");
  std::string err;
  if (int rc = mri::gguf_check(ggml_type, len, n_out * k_in, &err)) return fail(rc, "%s", err.c_str());
  mri_qmatrix* w = new mri_qmatrix{ctx->device, nullptr, nullptr, n_out, k_in, true};
  // Same zeroed slack after the rows as upload_bytes leaves.
  int rc = MRI_OK;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, n_out * k_in + kWeightPad);
  if (e == cudaSuccess) {
    w->data = static_cast<int8_t*>(p);
    e = cudaMemsetAsync(p, 0, n_out * k_in + kWeightPad, ctx->stream);
  }
  if (e == cudaSuccess) e = cudaMalloc(&p, n_out * sizeof(float) + kWeightPad);
  if (e == cudaSuccess) w->scales = static_cast<float*>(p);
  if (e != cudaSuccess) rc = cuda_fail(e, "weight allocation");
  if (rc == MRI_OK) {
    mri::GgufDst d;
    d.q = w->data;
    d.q_stride = k_in;
    d.scales = w->scales;
    rc = mri::gguf_to_device(ctx->stream, ggml_type, bytes, len, n_out, k_in, d, &err);
    if (rc != MRI_OK) fail(rc, "%s", err.c_str());
  }
  if (rc != MRI_OK) {
    if (w->data) cudaFree(w->data);
    if (w->scales) cudaFree(w->scales);
    delete w;
    return rc;
  }
  *out = w;
  return MRI_OK;
}

int mri_qmatrix_download(const mri_qmatrix* w, int8_t* data, float* scales) {
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null matrix");
  if ((!data && w->n_out * w->k_in) || (!scales && w->n_out))
    return fail(MRI_ERR_INVALID_ARGUMENT, "null output pointer");
  if (int rc = use_device(w->device)) return rc;
  if (w->n_out * w->k_in)
    MRI_CUDA_TRY(cudaMemcpy(data, w->data, w->n_out * w->k_in, cudaMemcpyDeviceToHost));
  if (w->n_out) MRI_CUDA_TRY(cudaMemcpy(scales, w->scales, w->n_out * 4, cudaMemcpyDeviceToHost));
  return MRI_OK;
}

int mri_gguf_dequant(mri_ctx* ctx, int ggml_type, const uint8_t* bytes, size_t len, size_t numel,
                     float* out_dev) {
  if (int rc = enter(ctx)) return rc;
  if (!out_dev && numel) return fail(MRI_ERR_INVALID_ARGUMENT, "null output pointer");
  mri::GgufDst d;
  d.f32 = out_dev;
  std::string err;
  // Viewed as rows of one block (32 values) so that the copy goes in steps.
  const size_t cols = numel % 32 == 0 && numel ? 32 : numel;
  const size_t rows = cols ? numel / cols : 0;
  if (int rc = mri::gguf_check(ggml_type, len, numel, &err)) return fail(rc, "%s", err.c_str());
  if (int rc = mri::gguf_to_device(ctx->stream, ggml_type, bytes, len, rows, cols, d, &err))
    return fail(rc, "%s", err.c_str());
  return MRI_OK;
}

int mri_q8_0_upload(mri_ctx* ctx, const uint8_t* bytes, size_t len, size_t n_out, size_t k_in,
                    mri_q8_0_matrix** out) {
  if (int rc = enter(ctx)) return rc;
  if (!out) return fail(MRI_ERR_INVALID_ARGUMENT, "null output pointer");
  // q8_direct.rs:81-104
  if (k_in % 32 != 0)
    return fail(MRI_ERR_INVALID_SHAPE, "Q8_0WeightMatrix: k_in=%zu is not a multiple of 32", k_in);
  const size_t expected = n_out * (k_in / 32) * 34;
  if (len != expected)
    return fail(MRI_ERR_INVALID_SHAPE,
                "Q8_0WeightMatrix: data.len()=%zu != expected %zu (n_out=%zu, n_blocks=%zu, "
                "block_size=34)",
                len, expected, n_out, k_in / 32);
  if (len && !bytes) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight pointer");
  mri_q8_0_matrix* w = new mri_q8_0_matrix{ctx->device, nullptr, n_out, k_in};
  if (int rc = upload_bytes(bytes, len, &w->data)) {
    delete w;
    return rc;
  }
  *out = w;
  return MRI_OK;
}

int mri_q8_0_free(mri_q8_0_matrix* w) {
  if (!w) return MRI_OK;
  use_device(w->device);
  cudaFree(w->data);
  delete w;
  return MRI_OK;
}

int mri_q4_0_upload(mri_ctx* ctx, const uint8_t* bytes, size_t len, size_t n_out, size_t k,
                    mri_q4_0_matrix** out) {
  if (int rc = enter(ctx)) return rc;
  if (!out) return fail(MRI_ERR_INVALID_ARGUMENT, "null output pointer");
  // q4_0.rs:121-140
  if (k % 32 != 0)
    return fail(MRI_ERR_INVALID_SHAPE,
                "matmul_q4_0_dequant: k=%zu must be a multiple of 32 (Q4_0 block size)", k);
  const size_t expected = n_out * (k / 32) * 18;
  if (len != expected)
    return fail(MRI_ERR_INVALID_SHAPE,
                "matmul_q4_0_dequant: weight_q4 has %zu bytes, expected %zu for shape [%zu, %zu]",
                len, expected, n_out, k);
  if (len && !bytes) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight pointer");
  mri_q4_0_matrix* w = new mri_q4_0_matrix{ctx->device, nullptr, n_out, k};
  if (int rc = upload_bytes(bytes, len, &w->data)) {
    delete w;
    return rc;
  }
  *out = w;
  return MRI_OK;
}

int mri_q4_0_free(mri_q4_0_matrix* w) {
  if (!w) return MRI_OK;
  use_device(w->device);
  cudaFree(w->data);
  delete w;
  return MRI_OK;
}

// ── quantizer ────────────────────────────────────────────────────────────────

int mri_quantize_symmetric(mri_ctx* ctx, const float* x_dev, size_t m, size_t k, int granularity,
                           int8_t* q_dev, float* scale_dev) {
  if (int rc = enter(ctx)) return rc;
  if (granularity != MRI_PER_TENSOR && granularity != MRI_PER_ROW)
    return fail(MRI_ERR_INVALID_ARGUMENT, "granularity must be MRI_PER_TENSOR or MRI_PER_ROW");
  if ((m * k && (!x_dev || !q_dev)) || !scale_dev)
    return fail(MRI_ERR_INVALID_ARGUMENT, "null device pointer");
  if (int rc = ensure_scratch(ctx, amax_bytes(m))) return rc;
  MRI_CUDA_TRY(mri::launch_quantize(ctx->dev, ctx->stream, x_dev, m, k, granularity, q_dev,
                                    scale_dev, reinterpret_cast<float*>(ctx->scratch), &ctx->ls, nullptr,
                                    0.0f, 0, ctx->d_sync, ctx->d_status));
  return MRI_OK;
}

// ── INT8 products ────────────────────────────────────────────────────────────

int mri_matmul_int8(mri_ctx* ctx, const int8_t* act_q_dev, size_t act_len, float act_scale,
                    const mri_qmatrix* w, size_t m, float* out_dev, int32_t* acc_dev) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (int rc = check_act_len("matmul_int8", act_len, m, w->k_in)) return rc;
  if (m * w->n_out && !out_dev) return fail(MRI_ERR_INVALID_ARGUMENT, "null output pointer");
  ActArgs a;
  a.xq = act_q_dev;
  a.mode = mri::ACT_I8_HOST_SCALE;
  a.scale_host = act_scale;
  return run_int8(ctx, a, w, m, out_dev, acc_dev);
}

int mri_matmul_int8_dscale(mri_ctx* ctx, const int8_t* act_q_dev, size_t act_len,
                           const float* act_scale_dev, int scale_per_row, const mri_qmatrix* w,
                           size_t m, float* out_dev, int32_t* acc_dev) {
  if (int rc = enter(ctx)) return rc;
  if (!w || !act_scale_dev) return fail(MRI_ERR_INVALID_ARGUMENT, "null argument");
  if (int rc = check_act_len("matmul_int8", act_len, m, w->k_in)) return rc;
  ActArgs a;
  a.xq = act_q_dev;
  a.mode = scale_per_row ? mri::ACT_I8_DEV_ROW_SCALE : mri::ACT_I8_DEV_SCALE;
  a.scale_dev = act_scale_dev;
  return run_int8(ctx, a, w, m, out_dev, acc_dev);
}

int mri_matmul_int8_from_f32_g(mri_ctx* ctx, const float* x_dev, size_t m, size_t k,
                               int granularity, const mri_qmatrix* w, float* out_dev) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (granularity != MRI_PER_TENSOR && granularity != MRI_PER_ROW)
    return fail(MRI_ERR_INVALID_ARGUMENT, "granularity must be MRI_PER_TENSOR or MRI_PER_ROW");
  if (int rc = check_k("matmul_int8_from_f32", m, k, w->k_in)) return rc;
  ActArgs a;
  a.x = x_dev;
  a.mode = granularity == MRI_PER_ROW ? mri::ACT_F32_PER_ROW : mri::ACT_F32_PER_TENSOR;
  return run_int8(ctx, a, w, m, out_dev, nullptr);
}

int mri_matmul_int8_from_f32(mri_ctx* ctx, const float* x_dev, size_t m, size_t k,
                             const mri_qmatrix* w, float* out_dev) {
  return mri_matmul_int8_from_f32_g(ctx, x_dev, m, k, MRI_PER_TENSOR, w, out_dev);
}

int mri_matmul_q8_0_direct(mri_ctx* ctx, const float* x_dev, size_t m, size_t k,
                           const mri_q8_0_matrix* w, float* out_dev) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (int rc = check_k("matmul_q8_0_direct", m, k, w->k_in)) return rc;
  return run_q8_0(ctx, x_dev, m, w, out_dev);
}

int mri_matmul_q4_0_dequant(mri_ctx* ctx, const float* x_dev, size_t m, size_t k,
                            const mri_q4_0_matrix* w, float* out_dev) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (int rc = check_k("matmul_q4_0_dequant", m, k, w->k)) return rc;
  return run_q4_0(ctx, x_dev, m, w, out_dev);
}

// ── host-buffer drop-ins ─────────────────────────────────────────────────────

int mri_host_quantize_symmetric(mri_ctx* ctx, const float* x, size_t m, size_t k, int granularity,
                                int8_t* q, float* scale) {
  if (int rc = enter(ctx)) return rc;
  if (granularity != MRI_PER_TENSOR && granularity != MRI_PER_ROW)
    return fail(MRI_ERR_INVALID_ARGUMENT, "granularity must be MRI_PER_TENSOR or MRI_PER_ROW");
  const size_t ns = granularity == MRI_PER_ROW ? m : 1;
  HostStage hs;
  if (int rc = host_stage(ctx, m * k * 4 + al(m * k), ns * 4, 0, std::max<size_t>(m, 1), 0, &hs))
    return rc;
  float* xd = reinterpret_cast<float*>(hs.in);
  int8_t* qd = reinterpret_cast<int8_t*>(hs.in + al(m * k * 4));
  if (m * k) MRI_CUDA_TRY(cudaMemcpyAsync(xd, x, m * k * 4, cudaMemcpyHostToDevice, ctx->stream));
  MRI_CUDA_TRY(mri::launch_quantize(ctx->dev, ctx->stream, xd, m, k, granularity, qd, hs.out,
                                    reinterpret_cast<float*>(ctx->scratch), &ctx->ls, nullptr, 0.0f, 0,
                                    ctx->d_sync, ctx->d_status));
  if (m * k) MRI_CUDA_TRY(cudaMemcpyAsync(q, qd, m * k, cudaMemcpyDeviceToHost, ctx->stream));
  if (ns) MRI_CUDA_TRY(cudaMemcpyAsync(scale, hs.out, ns * 4, cudaMemcpyDeviceToHost, ctx->stream));
  MRI_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return read_status(ctx);
}

int mri_host_matmul_int8(mri_ctx* ctx, const int8_t* act_q, size_t act_len, float act_scale,
                         const mri_qmatrix* w, size_t m, float* out, int32_t* acc) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (int rc = check_act_len("matmul_int8", act_len, m, w->k_in)) return rc;
  const size_t N = w->n_out;
  HostStage hs;
  if (int rc = host_stage(ctx, act_len, m * N * 4, acc ? m * N * 4 : 0, m, w->k_in, &hs)) return rc;
  if (act_len)
    MRI_CUDA_TRY(cudaMemcpyAsync(hs.in, act_q, act_len, cudaMemcpyHostToDevice, ctx->stream));
  ActArgs a;
  a.xq = reinterpret_cast<int8_t*>(hs.in);
  a.mode = mri::ACT_I8_HOST_SCALE;
  a.scale_host = act_scale;
  if (int rc = run_int8(ctx, a, w, m, hs.out, acc ? hs.acc : nullptr)) return rc;
  if (m * N) {
    MRI_CUDA_TRY(cudaMemcpyAsync(out, hs.out, m * N * 4, cudaMemcpyDeviceToHost, ctx->stream));
    if (acc) MRI_CUDA_TRY(cudaMemcpyAsync(acc, hs.acc, m * N * 4, cudaMemcpyDeviceToHost, ctx->stream));
  }
  MRI_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return read_status(ctx);
}

int mri_host_matmul_int8_from_f32(mri_ctx* ctx, const float* x, size_t m, size_t k,
                                  const mri_qmatrix* w, float* out) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (int rc = check_k("matmul_int8_from_f32", m, k, w->k_in)) return rc;
  const size_t N = w->n_out;
  HostStage hs;
  if (int rc = host_stage(ctx, m * k * 4, m * N * 4, 0, m, k, &hs)) return rc;

  if (m * k) MRI_CUDA_TRY(cudaMemcpyAsync(hs.in, x, m * k * 4, cudaMemcpyHostToDevice, ctx->stream));
  ActArgs a;
  a.x = reinterpret_cast<float*>(hs.in);
  a.mode = mri::ACT_F32_PER_TENSOR;
  if (int rc = run_int8(ctx, a, w, m, hs.out, nullptr)) return rc;
  if (int rc = copy_result(ctx, out, hs.out, m * N)) return rc;
  MRI_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return read_status(ctx);
}

int mri_host_matmul_q8_0_direct(mri_ctx* ctx, const float* x, size_t m, size_t k,
                                const mri_q8_0_matrix* w, float* out) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (int rc = check_k("matmul_q8_0_direct", m, k, w->k_in)) return rc;
  const size_t N = w->n_out;
  HostStage hs;
  if (int rc = host_stage(ctx, m * k * 4, m * N * 4, 0, m, k, &hs)) return rc;
  if (m * k) MRI_CUDA_TRY(cudaMemcpyAsync(hs.in, x, m * k * 4, cudaMemcpyHostToDevice, ctx->stream));
  if (int rc = run_q8_0(ctx, reinterpret_cast<float*>(hs.in), m, w, hs.out)) return rc;
  if (int rc = copy_result(ctx, out, hs.out, m * N)) return rc;
  MRI_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return read_status(ctx);
}

int mri_host_matmul_q4_0_dequant(mri_ctx* ctx, const float* x, size_t m, size_t k,
                                 const mri_q4_0_matrix* w, float* out) {
  if (int rc = enter(ctx)) return rc;
  if (!w) return fail(MRI_ERR_INVALID_ARGUMENT, "null weight handle");
  if (int rc = check_k("matmul_q4_0_dequant", m, k, w->k)) return rc;
  const size_t N = w->n_out;
  HostStage hs;
  // The reserved front of scratch holds run_q4_0's split activations (m rows
  // of 4k + 64 bytes).
  if (int rc = host_stage(ctx, m * k * 4, m * N * 4, 0, m, 4 * k + 64, &hs)) return rc;
  if (m * k) MRI_CUDA_TRY(cudaMemcpyAsync(hs.in, x, m * k * 4, cudaMemcpyHostToDevice, ctx->stream));
  if (int rc = run_q4_0(ctx, reinterpret_cast<float*>(hs.in), m, w, hs.out)) return rc;
  if (int rc = copy_result(ctx, out, hs.out, m * N)) return rc;
  MRI_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  return read_status(ctx);
}

int mri_int8_path(mri_ctx* ctx, size_t m, size_t n, size_t k) {
  if (!ctx) return -1;
  if (m <= 8 && m > 0 && mri::gemv_i8_tma_supported(ctx->dev, static_cast<int>(m), k)) return 0;
  if (mri::gemm_i8_tc_supported(ctx->dev, m, n, k)) return 2;  // (16-byte aligned activations)
  return 1;
}

int mri_int8_gemv_plan(mri_ctx* ctx, size_t m, size_t n, size_t k, int* plan) {
  if (int rc = enter(ctx)) return rc;
  if (!plan) return fail(MRI_ERR_INVALID_ARGUMENT, "null plan");
  if (m < 1 || m > 8 || !mri::gemv_i8_tma_supported(ctx->dev, static_cast<int>(m), k))
    return fail(MRI_ERR_INVALID_SHAPE, "no streaming GEMV for m=%zu, k=%zu", m, k);
  mri::GemvPlan p;
  MRI_CUDA_TRY(mri::gemv_i8_tma_plan(ctx->dev, static_cast<int>(m), n, k, &p));
  plan[0] = p.grid;
  plan[1] = p.ctas_per_sm;
  plan[2] = p.resident;
  plan[3] = p.stages;
  plan[4] = p.k_chunks;
  plan[5] = static_cast<int>(p.smem);
  // The register-prologue width of a per-tensor f32 input of this shape
  // (4 or 12 float4 per consumer thread; 0 = the input is quantized by the
  // quantizer kernels first and the GEMV streams int8 activations).
  plan[6] = p.vec;
  plan[7] = p.vec == 0 ? 1 : 0;
  return MRI_OK;
}

int mri_int8_gemm_plan(mri_ctx* ctx, size_t m, size_t n, size_t k, int* plan) {
  if (int rc = enter(ctx)) return rc;
  if (!plan) return fail(MRI_ERR_INVALID_ARGUMENT, "null plan");
  mri::GemmPlan p;
  if (mri::gemm_i8_tc_plan(ctx->dev, m, n, k, &p) != cudaSuccess)
    return fail(MRI_ERR_INVALID_SHAPE, "no tensor-core GEMM for m=%zu, n=%zu, k=%zu", m, n, k);
  plan[0] = p.bn;
  plan[1] = p.stages;
  plan[2] = p.bufs;
  plan[3] = p.grid;
  plan[4] = p.tiles;
  plan[5] = p.tiles_per_cta;
  plan[6] = p.pair;
  return MRI_OK;
}

}  // extern "C"
