// comm.cu — N-sharded INT8 products across the GPUs of one node.
//
// No reference counterpart: the reference runs on one host (rayon data
// parallelism over output rows, parallel.rs:308-346).  Here the output
// dimension N of a weight matrix is split across P ranks, one process per
// GPU: rank r holds rows [r*N/P, (r+1)*N/P) of W and their scales, computes
// its [M, N/P] slice with the same kernels (and therefore the same INT32 sums
// and f32 epilogue) as the unsharded product, and an NCCL all-gather over
// NVLink assembles the full [M, N] output on every rank.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2): a process that
// already loaded NCCL (torch.distributed) shares that library, and the
// shared object stays loadable on machines without NCCL.  Communicators are
// created non-blocking, so every host-side wait has a deadline after which
// the communicator is aborted and the call returns MRI_ERR_TIMEOUT.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "common.cuh"
#include "internal.h"
#include "mri_gpu.h"

namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      api.why = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    auto sym = [&](const char* name) { return dlsym(h, name); };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.init_rank_config = reinterpret_cast<decltype(api.init_rank_config)>(sym("ncclCommInitRankConfig"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(sym("ncclCommDestroy"));
    api.abort = reinterpret_cast<decltype(api.abort)>(sym("ncclCommAbort"));
    api.async_error = reinterpret_cast<decltype(api.async_error)>(sym("ncclCommGetAsyncError"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.ok = api.get_unique_id && api.init_rank_config && api.destroy && api.abort &&
             api.async_error && api.all_gather && api.error_string;
    if (!api.ok) api.why = "libnccl.so.2 lacks a required symbol (NCCL >= 2.14 needed)";
  });
  return api;
}

constexpr int kMaxChunks = 8;

const char* nccl_str(ncclResult_t r) { return nccl().error_string ? nccl().error_string(r) : "?"; }

}  // namespace

struct mri_comm {
  mri_ctx* ctx = nullptr;
  ncclComm_t comm = nullptr;
  int rank = 0, size = 1;
  int timeout_ms = 60000;
  bool aborted = false;
  cudaStream_t side = nullptr;  // all-gathers and unshard copies of chunked products
  cudaEvent_t chunk_ready[kMaxChunks] = {};
  cudaEvent_t side_done = nullptr;
  float* gather = nullptr;  // rank-major staging [chunk][P][rows][N/P]
  size_t gather_bytes = 0;
};

namespace {

using Clock = std::chrono::steady_clock;

int abort_comm(mri_comm* c, const char* what) {
  if (!c->aborted && c->comm) nccl().abort(c->comm);
  c->aborted = true;
  c->comm = nullptr;
  return mri::set_error(MRI_ERR_TIMEOUT, "%s: no progress within %d ms; communicator aborted", what,
                        c->timeout_ms);
}

// Completes a non-blocking NCCL call: ncclInProgress means the call is still
// being set up on the host; poll until it is done, fails, or the deadline passes.
int settle(mri_comm* c, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return MRI_OK;
  if (r != ncclInProgress) return mri::set_error(MRI_ERR_COMM, "%s: %s", what, nccl_str(r));
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  for (;;) {
    ncclResult_t st = ncclInProgress;
    const ncclResult_t q = nccl().async_error(c->comm, &st);
    if (q != ncclSuccess) return mri::set_error(MRI_ERR_COMM, "%s: %s", what, nccl_str(q));
    if (st == ncclSuccess) return MRI_OK;
    if (st != ncclInProgress) return mri::set_error(MRI_ERR_COMM, "%s: %s", what, nccl_str(st));
    if (Clock::now() > deadline) return abort_comm(c, what);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int cuda_err(cudaError_t e, const char* what) {
  return mri::set_error(MRI_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define COMM_CUDA_TRY(expr)                             \
  do {                                                  \
    cudaError_t _e = (expr);                            \
    if (_e != cudaSuccess) return cuda_err(_e, #expr);  \
  } while (0)

// g: [P][rows][ns] (rank-major) -> out rows [rows][P*ns] at row stride ld.
__global__ void unshard_kernel(const float* __restrict__ g, int P, size_t rows, size_t ns,
                               float* __restrict__ out, size_t ld) {
  const size_t width = static_cast<size_t>(P) * ns;
  const size_t total = rows * width;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  if ((ns & 3) == 0 && (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(g) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
    const size_t ns4 = ns / 4, w4 = width / 4;
    for (size_t t = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; t < total / 4; t += stride) {
      const size_t i = t / w4, c = t - i * w4, p = c / ns4, j = c - p * ns4;
      const float4 v = mri::ld_act(reinterpret_cast<const float4*>(g + (p * rows + i) * ns) + j);
      reinterpret_cast<float4*>(out + i * ld)[c] = v;
    }
  } else {
    for (size_t t = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; t < total; t += stride) {
      const size_t i = t / width, c = t - i * width, p = c / ns, j = c - p * ns;
      out[i * ld + c] = g[(p * rows + i) * ns + j];
    }
  }
}

int launch_unshard(mri_comm* c, cudaStream_t st, const float* g, size_t rows, size_t ns, float* out,
                   size_t ld) {
  const size_t n = rows * ns * c->size;
  const int threads = 256;
  const int blocks = static_cast<int>(std::max<size_t>(
      1, std::min<size_t>((n / 4 + threads - 1) / threads, static_cast<size_t>(c->ctx->dev.sm_count) * 8)));
  unshard_kernel<<<blocks, threads, 0, st>>>(g, c->size, rows, ns, out, ld);
  c->ctx->ls.launches++;
  COMM_CUDA_TRY(cudaGetLastError());
  return MRI_OK;
}

int ensure_gather(mri_comm* c, size_t bytes) {
  if (bytes <= c->gather_bytes) return MRI_OK;
  if (c->gather) {
    COMM_CUDA_TRY(cudaStreamSynchronize(c->ctx->stream));
    COMM_CUDA_TRY(cudaStreamSynchronize(c->side));
    COMM_CUDA_TRY(cudaFree(c->gather));
    c->gather = nullptr;
    c->gather_bytes = 0;
  }
  COMM_CUDA_TRY(cudaMalloc(&c->gather, bytes));
  c->gather_bytes = bytes;
  return MRI_OK;
}

// Row chunks of an M-row sharded product: each chunk's all-gather overlaps the
// next chunk's GEMM.  MRI_SHARD_CHUNKS overrides the count.
int chunk_count(size_t m) {
  int n = m >= 1024 ? 4 : (m >= 256 ? 2 : 1);
  if (const char* e = std::getenv("MRI_SHARD_CHUNKS")) n = std::atoi(e);
  n = std::max(1, std::min(n, kMaxChunks));
  return static_cast<int>(std::min<size_t>(n, std::max<size_t>(1, m)));
}

int check_comm(mri_comm* c) {
  if (!c) return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "null communicator");
  if (c->aborted) return mri::set_error(MRI_ERR_COMM, "communicator was aborted after a timeout");
  return MRI_OK;
}

}  // namespace

extern "C" {

int mri_comm_available(void) { return nccl().ok ? 1 : 0; }

int mri_comm_unique_id(uint8_t* id) {
  if (!id) return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "null id buffer");
  if (!nccl().ok) return mri::set_error(MRI_ERR_COMM, "%s", nccl().why.c_str());
  static_assert(sizeof(ncclUniqueId) == MRI_COMM_ID_BYTES, "NCCL unique id size");
  ncclUniqueId u;
  const ncclResult_t r = nccl().get_unique_id(&u);
  if (r != ncclSuccess) return mri::set_error(MRI_ERR_COMM, "ncclGetUniqueId: %s", nccl_str(r));
  std::memcpy(id, &u, sizeof(u));
  return MRI_OK;
}

int mri_shard_rows(size_t n, int nranks, int rank, size_t* row_begin, size_t* row_end) {
  if (!row_begin || !row_end) return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "null output");
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "rank %d of %d", rank, nranks);
  if (n % static_cast<size_t>(nranks))
    return mri::set_error(MRI_ERR_INVALID_SHAPE, "n_out=%zu is not divisible by %d ranks", n, nranks);
  const size_t ns = n / nranks;
  *row_begin = ns * rank;
  *row_end = ns * (rank + 1);
  return MRI_OK;
}

int mri_comm_create(mri_ctx* ctx, const uint8_t* id, int nranks, int rank, int timeout_ms,
                    mri_comm** out) {
  if (!ctx || !id || !out) return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "rank %d of %d", rank, nranks);
  if (!nccl().ok) return mri::set_error(MRI_ERR_COMM, "%s", nccl().why.c_str());
  COMM_CUDA_TRY(cudaSetDevice(ctx->device));
  mri_comm* c = new mri_comm();
  c->ctx = ctx;
  c->rank = rank;
  c->size = nranks;
  c->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  cudaError_t e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
  for (int i = 0; i < kMaxChunks && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&c->chunk_ready[i], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->side_done, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    mri_comm_destroy(c);
    return cuda_err(e, "comm streams/events");
  }
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  const ncclResult_t r = nccl().init_rank_config(&c->comm, nranks, u, rank, &cfg);
  if (int rc = (c->comm ? settle(c, r, "ncclCommInitRankConfig")
                        : mri::set_error(MRI_ERR_COMM, "ncclCommInitRankConfig: %s", nccl_str(r)))) {
    mri_comm_destroy(c);
    return rc;
  }
  *out = c;
  return MRI_OK;
}

int mri_comm_destroy(mri_comm* c) {
  if (!c) return MRI_OK;
  cudaSetDevice(c->ctx->device);
  if (c->comm) {
    // Drain our work first; a communicator that cannot finish is aborted.
    if (mri_comm_wait(c) == MRI_OK && c->comm) nccl().destroy(c->comm);
  }
  if (c->gather) cudaFree(c->gather);
  for (auto& ev : c->chunk_ready)
    if (ev) cudaEventDestroy(ev);
  if (c->side_done) cudaEventDestroy(c->side_done);
  if (c->side) cudaStreamDestroy(c->side);
  delete c;
  return MRI_OK;
}

int mri_comm_rank(const mri_comm* c, int* rank, int* nranks) {
  if (!c || !rank || !nranks) return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "null argument");
  *rank = c->rank;
  *nranks = c->size;
  return MRI_OK;
}

int mri_comm_wait(mri_comm* c) {
  if (!c) return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "null communicator");
  COMM_CUDA_TRY(cudaSetDevice(c->ctx->device));
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  for (cudaStream_t st : {c->ctx->stream, c->side}) {
    for (;;) {
      const cudaError_t q = cudaStreamQuery(st);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return cuda_err(q, "cudaStreamQuery");
      if (c->comm) {
        ncclResult_t st_async = ncclSuccess;
        nccl().async_error(c->comm, &st_async);
        if (st_async != ncclSuccess && st_async != ncclInProgress) {
          nccl().abort(c->comm);
          c->comm = nullptr;
          c->aborted = true;
          return mri::set_error(MRI_ERR_COMM, "NCCL error: %s", nccl_str(st_async));
        }
      }
      if (Clock::now() > deadline) return abort_comm(c, "mri_comm_wait");
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  }
  return MRI_OK;
}

int mri_sharded_matmul_int8_from_f32(mri_comm* c, const float* x_dev, size_t m, size_t k,
                                     const mri_qmatrix* w_shard, size_t n_total, float* out_dev) {
  if (int rc = check_comm(c)) return rc;
  if (!w_shard) return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "null weight shard");
  const int P = c->size, r = c->rank;
  if (n_total % static_cast<size_t>(P))
    return mri::set_error(MRI_ERR_INVALID_SHAPE, "n_total=%zu is not divisible by %d ranks", n_total, P);
  const size_t ns = n_total / P;
  if (w_shard->n_out != ns)
    return mri::set_error(MRI_ERR_SHAPE_MISMATCH, "expected a shard of %zu rows, got %zu", ns,
                          w_shard->n_out);
  if (k != w_shard->k_in)
    return mri::set_error(MRI_ERR_SHAPE_MISMATCH, "expected [%zu, %zu], got [%zu, %zu]", m,
                          w_shard->k_in, m, k);
  if (m == 0 || n_total == 0) return MRI_OK;
  if (!x_dev || !out_dev) return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "null buffer");
  mri_ctx* ctx = c->ctx;
  COMM_CUDA_TRY(cudaSetDevice(ctx->device));
  cudaStream_t st = ctx->stream;
  const NcclApi& api = nccl();

  if (m == 1) {
    // One row: the rank-major gather layout is the output layout.
    float* slot = out_dev + r * ns;
    mri::ActArgs a;
    a.x = x_dev;
    a.mode = mri::ACT_F32_PER_TENSOR;
    if (int rc = mri::matmul_int8_act(ctx, a, w_shard, 1, slot)) return rc;
    return settle(c, api.all_gather(slot, out_dev, ns, ncclFloat32, c->comm, st), "ncclAllGather");
  }

  // Quantize the whole input once (per-tensor scale over all M*K values, as
  // the unsharded call), then run row chunks: chunk j's slice goes to its slot
  // of the staging buffer on the compute stream, and its all-gather and
  // unshard copy run on the side stream while chunk j+1 computes.
  const int chunks = m <= 8 ? 1 : chunk_count(m);
  if (int rc = ensure_gather(c, m * n_total * sizeof(float))) return rc;
  int8_t* q = nullptr;
  float* scale_dev = nullptr;
  mri::ActArgs a;
  if (m > 8) {
    if (int rc = mri::quantize_to_scratch(ctx, x_dev, m, k, &q, &scale_dev)) return rc;
  } else {
    a.x = x_dev;
    a.mode = mri::ACT_F32_PER_TENSOR;
  }
  const size_t per = (m + chunks - 1) / chunks;
  for (int j = 0; j < chunks; ++j) {
    const size_t m0 = per * j;
    if (m0 >= m) break;
    const size_t mc = std::min(per, m - m0);
    float* base = c->gather + m0 * n_total;  // [P][mc][ns] for this chunk
    float* slot = base + r * mc * ns;
    if (m > 8) {
      a.xq = q + m0 * k;
      a.mode = mri::ACT_I8_DEV_SCALE;
      a.scale_dev = scale_dev;
    }
    if (int rc = mri::matmul_int8_act(ctx, a, w_shard, mc, slot)) return rc;
    COMM_CUDA_TRY(cudaEventRecord(c->chunk_ready[j], st));
    COMM_CUDA_TRY(cudaStreamWaitEvent(c->side, c->chunk_ready[j], 0));
    if (int rc = settle(c, api.all_gather(slot, base, mc * ns, ncclFloat32, c->comm, c->side),
                        "ncclAllGather"))
      return rc;
    if (int rc = launch_unshard(c, c->side, base, mc, ns, out_dev + m0 * n_total, n_total)) return rc;
  }
  COMM_CUDA_TRY(cudaEventRecord(c->side_done, c->side));
  COMM_CUDA_TRY(cudaStreamWaitEvent(st, c->side_done, 0));
  return MRI_OK;
}

}  // extern "C"
