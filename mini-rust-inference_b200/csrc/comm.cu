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
// With MRI_SHARD_PEER=1, for m <= 8 (decode) the gather runs over peer memory
// instead: every rank maps every other rank's staging buffer and arrival
// counter (CUDA IPC over NVLink), the GEMV epilogue writes its output rows to
// all ranks and counts itself in on every rank, and a small collect kernel
// waits (bounded) for all ranks before copying the assembled result out.  No
// collective launch.  The ranks agree collectively whether the mappings work;
// if any rank cannot map them, all use the NCCL path.
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
#include <vector>

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
  // Peer-memory gather (m <= 8).
  bool peer_tried = false, peer_ok = false;
  float* stage = nullptr;                 // local staging [2][stage_half]
  size_t stage_half = 0;
  unsigned long long* ctrs = nullptr;     // [0] arrival counter; call state from byte 128 (gemv.cu)
  float* peer_stage[mri::EpiArgs::kMaxRanks] = {};
  unsigned long long* peer_ctr[mri::EpiArgs::kMaxRanks] = {};
  std::vector<void*> retired;             // earlier staging buffers (peers may still map them)
  std::vector<void*> opened;              // peer mappings to close
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

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Second half of a gathered GEMM (mri::GemmOut): waits (bounded) until every
// rank's CTAs have counted themselves in, then copies the other ranks'
// columns [0, c0) and [c0 + ns, n_total) of this call's staging half into
// out [M][n_total].  Every block waits on its own; the copy is flat over
// M * (n_total - ns) elements, float4-wide when the layout allows.
__global__ void __launch_bounds__(256) gather_collect_cols_kernel(
    const unsigned long long* ctr, const unsigned long long* call, const float* stage, size_t half, size_t M,
    size_t n_total, size_t c0, size_t ns, float* out, int* status) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const unsigned long long target = __ldcg(call);
    int ok = 1;
    const long long t0 = clock64();
    while (ld_acquire_sys(ctr) < target) {
      if (clock64() - t0 > mri::kWaitBudgetClocks) {
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
  const float* src = stage + ((__ldcg(call + 2) - 1) & 1) * half;
  const size_t w = n_total - ns;  // columns copied per row
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w % 4 == 0 && c0 % 4 == 0 && n_total % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const size_t w4 = w / 4, c04 = c0 / 4, ns4 = ns / 4, n4 = n_total / 4;
    for (size_t i = tid; i < M * w4; i += stride) {
      const size_t r = i / w4, j = i - r * w4;
      const size_t col4 = j < c04 ? j : j + ns4;
      reinterpret_cast<float4*>(out)[r * n4 + col4] = __ldcg(reinterpret_cast<const float4*>(src) + r * n4 + col4);
    }
    return;
  }
  for (size_t i = tid; i < M * w; i += stride) {
    const size_t r = i / w, j = i - r * w;
    const size_t col = j < c0 ? j : j + ns;
    out[r * n_total + col] = __ldcg(src + r * n_total + col);
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
// next chunk's GEMM.
int chunk_count(size_t m) {
  int n = m >= 1024 ? 4 : (m >= 256 ? 2 : 1);
  n = std::max(1, std::min(n, kMaxChunks));
  return static_cast<int>(std::min<size_t>(n, std::max<size_t>(1, m)));
}

int check_comm(mri_comm* c) {
  if (!c) return mri::set_error(MRI_ERR_INVALID_ARGUMENT, "null communicator");
  if (c->aborted) return mri::set_error(MRI_ERR_COMM, "communicator was aborted after a timeout");
  return MRI_OK;
}

// All-gathers `bytes` bytes of host data from every rank (through a device
// buffer and NCCL on the context stream); synchronizes the stream.
int exchange(mri_comm* c, const void* mine, size_t bytes, std::vector<uint8_t>* all) {
  void* d = nullptr;
  COMM_CUDA_TRY(cudaMalloc(&d, bytes * c->size));
  int rc = MRI_OK;
  cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(d) + bytes * c->rank, mine, bytes,
                                  cudaMemcpyHostToDevice, c->ctx->stream);
  if (e != cudaSuccess) rc = cuda_err(e, "exchange upload");
  if (!rc)
    rc = settle(c, nccl().all_gather(static_cast<uint8_t*>(d) + bytes * c->rank, d, bytes, ncclUint8,
                                     c->comm, c->ctx->stream),
                "ncclAllGather (peer setup)");
  if (!rc) rc = mri_comm_wait(c);
  all->resize(bytes * c->size);
  if (!rc) {
    e = cudaMemcpy(all->data(), d, bytes * c->size, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) rc = cuda_err(e, "exchange download");
  }
  cudaFree(d);
  return rc;
}

// Collective: makes sure every rank's staging holds `half` floats per half and
// every rank maps every other rank's staging and counters.  Sets peer_ok to
// the ranks' joint verdict.  Called with the same `half` on every rank (the
// ranks issue the same sequence of sharded calls).
int ensure_peer(mri_comm* c, size_t half) {
  if (c->peer_tried && (!c->peer_ok || half <= c->stage_half)) return MRI_OK;
  c->peer_tried = true;
  const bool first = c->ctrs == nullptr;
  half = std::max(half, c->stage_half * 2);
  struct Msg {
    int ok;
    int pad;
    cudaIpcMemHandle_t stage, ctrs;
  } mine{};
  float* stage = nullptr;
  mine.ok = 1;
  if (cudaMalloc(&stage, 2 * half * sizeof(float)) != cudaSuccess) {
    cudaGetLastError();
    stage = nullptr;
    mine.ok = 0;
  }
  if (mine.ok && first) {
    void* ctrs = nullptr;
    if (cudaMalloc(&ctrs, 512) != cudaSuccess || cudaMemset(ctrs, 0, 512) != cudaSuccess) {
      cudaGetLastError();
      mine.ok = 0;
    } else {
      c->ctrs = static_cast<unsigned long long*>(ctrs);
    }
  }
  if (mine.ok && c->size > 1) {
    if (cudaIpcGetMemHandle(&mine.stage, stage) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine.ctrs, c->ctrs) != cudaSuccess) {
      cudaGetLastError();
      mine.ok = 0;
    }
  }
  std::vector<uint8_t> all;
  if (int rc = c->size > 1 ? exchange(c, &mine, sizeof(Msg), &all) : MRI_OK) {
    if (stage) cudaFree(stage);
    c->peer_ok = false;
    return rc;
  }
  bool every = mine.ok != 0;
  for (int p = 0; p < c->size && c->size > 1; ++p)
    every = every && reinterpret_cast<const Msg*>(all.data())[p].ok;
  // Map the other ranks' buffers, then agree again on whether that worked.
  int mapped = every ? 1 : 0;
  float* new_stage[mri::EpiArgs::kMaxRanks] = {};
  unsigned long long* new_ctr[mri::EpiArgs::kMaxRanks] = {};
  std::vector<void*> opened_now;
  if (every) {
    for (int p = 0; p < c->size; ++p) {
      if (p == c->rank) {
        new_stage[p] = stage;
        new_ctr[p] = c->ctrs;
        continue;
      }
      const Msg& m = reinterpret_cast<const Msg*>(all.data())[p];
      void* ps = nullptr;
      void* pc = c->peer_ctr[p];
      if (cudaIpcOpenMemHandle(&ps, m.stage, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        mapped = 0;
        break;
      }
      opened_now.push_back(ps);
      if (!pc) {
        if (cudaIpcOpenMemHandle(&pc, m.ctrs, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
          cudaGetLastError();
          mapped = 0;
          break;
        }
        opened_now.push_back(pc);
      }
      new_stage[p] = static_cast<float*>(ps);
      new_ctr[p] = static_cast<unsigned long long*>(pc);
    }
  }
  if (c->size > 1) {
    std::vector<uint8_t> verdicts;
    if (int rc = exchange(c, &mapped, sizeof(int), &verdicts)) {
      for (void* v : opened_now) cudaIpcCloseMemHandle(v);
      if (stage) cudaFree(stage);
      c->peer_ok = false;
      return rc;
    }
    for (int p = 0; p < c->size; ++p) mapped = mapped && reinterpret_cast<const int*>(verdicts.data())[p];
  }
  if (!mapped) {
    for (void* v : opened_now) cudaIpcCloseMemHandle(v);
    if (stage) cudaFree(stage);
    c->peer_ok = false;
    return MRI_OK;
  }
  if (c->stage) c->retired.push_back(c->stage);
  c->stage = stage;
  c->stage_half = half;
  for (int p = 0; p < c->size; ++p) {
    c->peer_stage[p] = new_stage[p];
    c->peer_ctr[p] = new_ctr[p];
  }
  c->opened.insert(c->opened.end(), opened_now.begin(), opened_now.end());
  c->peer_ok = true;
  return MRI_OK;
}

}  // namespace

namespace mri {
cudaError_t launch_gather_collect_cols(const DeviceInfo& dev, cudaStream_t st, const GemmOut& g, size_t M,
                                       size_t ns, float* out_full, int* status, LaunchStats* ls) {
  const size_t n_total = ns * static_cast<size_t>(g.ranks);
  const size_t work = M * (n_total - ns) / 4 + 1;
  const int grid = static_cast<int>(std::max<size_t>(1, std::min<size_t>(static_cast<size_t>(dev.sm_count) * 4,
                                                                         (work + 255) / 256)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dev.opt.pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gather_collect_cols_kernel,
                                     static_cast<const unsigned long long*>(g.ctr[g.rank]),
                                     static_cast<const unsigned long long*>(g.seq),
                                     static_cast<const float*>(g.stage[g.rank]), g.half, M, n_total, g.col0, ns,
                                     out_full, status);
  if (ls) ls->launches++;
  return e;
}
}  // namespace mri

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
  for (void* v : c->opened) cudaIpcCloseMemHandle(v);
  for (void* v : c->retired) cudaFree(v);
  if (c->stage) cudaFree(c->stage);
  if (c->ctrs) cudaFree(c->ctrs);
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
  // A peer-gather kernel that gave up waiting for the other ranks leaves the
  // arrival counts inconsistent: the communicator cannot be used again.
  if (int rc = mri_ctx_check_device_status(c->ctx)) {
    if (c->comm) nccl().abort(c->comm);
    c->comm = nullptr;
    c->aborted = true;
    return rc;
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

  if (P == 1) {  // the shard is the whole matrix: nothing to gather
    mri::ActArgs a;
    a.x = x_dev;
    a.mode = mri::ACT_F32_PER_TENSOR;
    return mri::matmul_int8_act(ctx, a, w_shard, m, out_dev);
  }

  mri::GemvPlan plan;
  const bool gather_fits =
      m <= 8 && mri::stream_gemv_ok(ctx, m, w_shard) &&
      mri::gemv_i8_tma_plan(ctx->dev, static_cast<int>(m), ns, k, &plan, -1, 2) == cudaSuccess &&
      ((ns + plan.grid - 1) / plan.grid) * m <= 1024;
  // MRI_OPT_SHARD_PEER = 1 selects the peer-memory gather for m <= 8 too.
  // Not the default: on 2 B200s it measured 34.1 us per 70B gate/up shard
  // call against 32.2 us for GEMV + NCCL all-gather (the shard GEMV alone:
  // 19.8 us).
  if (gather_fits && c->ctx->dev.opt.shard_peer == 1) {
    if (int rc = ensure_peer(c, m * n_total)) return rc;
    if (c->peer_ok) {
      mri::EpiArgs e;
      e.mode = mri::EPI_GATHER;
      for (int p = 0; p < P; ++p) {
        e.g_stage[p] = c->peer_stage[p];
        e.g_ctr[p] = c->peer_ctr[p];
      }
      e.g_seq = c->ctrs + 16;  // call state on the lines after the arrival counter
      e.g_half = c->stage_half;
      e.g_ntotal = n_total;
      e.g_ranks = P;
      e.g_rank = r;
      e.g_out = out_dev;
      return mri::matmul_int8_gather(ctx, x_dev, m, k, w_shard, e);
    }
  }

  // More rows, peer-memory path (the default, MRI_OPT_SHARD_PEER 1 or 2):
  // one tensor-core GEMM writes its tiles to every rank (its own columns
  // straight into out, the other ranks' staging over NVLink as each tile
  // completes), then a collect kernel waits for the other ranks and copies
  // their columns out of this rank's staging.  On 2 B200s at the 70B FFN
  // shapes (M = 2048): gate/up 0.358 ms against 0.651 ms with the chunked
  // NCCL all-gather, down 0.408 against 0.582 ms.
  if (m > 8 && c->ctx->dev.opt.shard_peer != 0 &&
      mri::gemm_i8_tc_supported(ctx->dev, m, ns, k) &&
      (reinterpret_cast<uintptr_t>(w_shard->data) & 15) == 0) {
    if (int rc = ensure_peer(c, m * n_total)) return rc;
    if (c->peer_ok) {
      int8_t* q = nullptr;
      float* scale_dev = nullptr;
      if (int rc = mri::quantize_to_scratch(ctx, x_dev, m, k, &q, &scale_dev)) return rc;
      mri::GemmOut g;
      g.out = out_dev + r * ns;
      g.ldo = n_total;
      g.ranks = P;
      g.rank = r;
      g.half = c->stage_half;
      g.col0 = r * ns;
      for (int p = 0; p < P; ++p) {
        g.stage[p] = c->peer_stage[p];
        g.ctr[p] = c->peer_ctr[p];
      }
      g.seq = c->ctrs + 16;  // call state on the lines after the arrival counter
      COMM_CUDA_TRY(mri::launch_gemm_i8_tc(ctx->dev, st, q, scale_dev, 0, w_shard->data, w_shard->scales, m, ns,
                                           k, nullptr, nullptr, ctx->d_status, &ctx->ls, nullptr, &g));
      COMM_CUDA_TRY(mri::launch_gather_collect_cols(ctx->dev, st, g, m, ns, out_dev, ctx->d_status, &ctx->ls));
      return MRI_OK;
    }
  }

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
