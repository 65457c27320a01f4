// noalloc.cu — an allocation-free variant of matmul_int8_from_f32 (per-tensor
// activation quantization, then the streaming GEMV for 1..8 rows or the
// tcgen05 GEMM for more).
//
// Who needs it: callers that must not allocate device memory at call time —
// code running inside a memory pool they do not own, an embedding runtime
// that forbids cudaMalloc/cudaFree on its threads, or a stream that is being
// fed by a framework whose allocator would otherwise be bypassed.  The
// regular entry points keep their scratch in a per-context buffer that grows
// with cudaMalloc; this one keeps it in a fixed, file-scope device array.
//
// The array holds the quantized activations (up to kNoAllocMaxActBytes) plus
// a small header (absmax accumulator, activation scale, wait-status word).
// Every GPU that loads this library holds the array until the process exits.
// The status word is sticky: a bounded device-side wait that gives up writes
// MRI_ERR_TIMEOUT there, and it stays set until mri_noalloc_check_status reads
// and clears it.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "internal.h"
#include "mri_gpu.h"

namespace {

// Header: maxima area (kQuantPartials floats), activation scale, status word.
constexpr size_t kHeaderBytes = mri::kQuantPartials * sizeof(float) + 256;
constexpr size_t kNoAllocMaxActBytes = MRI_NOALLOC_MAX_ACT_BYTES;

// Layout: [0, 4096) per-block absmax partials (f32), then the activation
// scale (f32) and the status word (i32), then the quantized activations at
// kHeaderBytes.
constexpr size_t kScaleOffset = mri::kQuantPartials * sizeof(float);
constexpr size_t kStatusOffset = kScaleOffset + 8;
constexpr size_t kSyncOffset = kScaleOffset + 16;  // two words: the quantizer's grid barrier
__device__ __align__(256) uint8_t g_noalloc_scratch[kHeaderBytes + kNoAllocMaxActBytes];

constexpr int kMaxDevices = 64;

struct DeviceSetup {
  bool ready = false;
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  mri::DeviceInfo dev;
};

std::mutex g_setup_mu;
DeviceSetup g_setup[kMaxDevices];
thread_local std::string g_noalloc_error;

int fail(int code, const char* msg) {
  g_noalloc_error = msg;
  return code;
}

// Once per device, with that device current: resolve the device address of
// the file-scope array (in host code its name is only a stand-in) and read
// the device properties the launchers need, then clear the status word on
// `st`.  Allocation-free.
int setup_device(int device, cudaStream_t st, DeviceSetup** out) {
  if (device < 0 || device >= kMaxDevices) return fail(MRI_ERR_CUDA, "device index out of range");
  std::lock_guard<std::mutex> lock(g_setup_mu);
  DeviceSetup& s = g_setup[device];
  if (!s.ready) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return fail(MRI_ERR_CUDA, cudaGetErrorString(e));
    int sms = 0, major = 0, minor = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device)) != cudaSuccess)
      return fail(MRI_ERR_CUDA, cudaGetErrorString(e));
    if (major != 10) return fail(MRI_ERR_CUDA, "device is not sm_100 (this library is built for sm_100a)");
    if ((e = cudaMemsetAsync(static_cast<uint8_t*>(ptr) + kStatusOffset, 0, kSyncOffset + 8 - kStatusOffset,
                             st)) != cudaSuccess)
      return fail(MRI_ERR_CUDA, cudaGetErrorString(e));
    s.scratch = static_cast<uint8_t*>(ptr);
    s.dev.device = device;
    s.dev.sm_count = sms;
    s.dev.cc_major = major;
    s.dev.cc_minor = minor;
    s.ready = true;
  }
  *out = &s;
  return MRI_OK;
}

}  // namespace

extern "C" {

const char* mri_noalloc_last_error(void) { return g_noalloc_error.c_str(); }

int mri_matmul_int8_from_f32_noalloc(const float* x_dev, size_t m, size_t k, const int8_t* w_dev,
                                     const float* w_scales_dev, size_t n, float* out_dev,
                                     void* cuda_stream) {
  g_noalloc_error.clear();
  // Size checks first, written so that no product can wrap around.
  if (m > 0 && (k > kNoAllocMaxActBytes || m > kNoAllocMaxActBytes / k)) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "matmul_int8_from_f32_noalloc: m=%zu x k=%zu activation bytes exceed the fixed scratch of "
             "%zu bytes",
             m, k, kNoAllocMaxActBytes);
    return fail(MRI_ERR_INVALID_ARGUMENT, buf);
  }
  if (m == 0 || n == 0) return MRI_OK;
  if (!x_dev || !w_dev || !w_scales_dev || !out_dev)
    return fail(MRI_ERR_INVALID_ARGUMENT, "null device pointer");
  if (k < 16 || k % 16 != 0)
    return fail(MRI_ERR_INVALID_SHAPE, "matmul_int8_from_f32_noalloc: k must be a positive multiple of 16");
  if (reinterpret_cast<uintptr_t>(w_dev) & 15)
    return fail(MRI_ERR_INVALID_ARGUMENT, "weights must be 16-byte aligned");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return fail(MRI_ERR_CUDA, cudaGetErrorString(e));
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  DeviceSetup* s = nullptr;
  if (int rc = setup_device(device, st, &s)) return rc;
  float* amax = reinterpret_cast<float*>(s->scratch);
  float* scale = reinterpret_cast<float*>(s->scratch + kScaleOffset);
  int* status = reinterpret_cast<int*>(s->scratch + kStatusOffset);
  int8_t* xq = reinterpret_cast<int8_t*>(s->scratch + kHeaderBytes);
  const bool gemv = m <= 8 && mri::gemv_i8_tma_supported(s->dev, static_cast<int>(m), k);
  if (!gemv && !mri::gemm_i8_tc_supported(s->dev, m, n, k))
    return fail(MRI_ERR_CUDA, "tensor-core GEMM unavailable on this device/driver");
  mri::ActArgs act;
  act.x = x_dev;
  act.mode = mri::ACT_F32_PER_TENSOR;
  // 1..8 rows: the streaming GEMV, which quantizes an input that fits its
  // register prologue itself and needs no scratch; a longer input is
  // quantized into the array first.  More rows: quantizer, then the
  // tensor-core GEMM.
  if (gemv && mri::reg_vec(static_cast<int>(m), k, &act) != 0) {
    e = mri::launch_gemv_i8_tma(s->dev, st, static_cast<int>(m), w_dev, w_scales_dev, n, k, act, out_dev,
                                nullptr, status, nullptr);
    return e == cudaSuccess ? MRI_OK : fail(MRI_ERR_CUDA, cudaGetErrorString(e));
  }
  unsigned* sync = reinterpret_cast<unsigned*>(s->scratch + kSyncOffset);
  if ((e = mri::launch_quantize(s->dev, st, x_dev, m, k, /*per_row=*/0, xq, scale, amax, nullptr, nullptr,
                                0.0f, 0, sync, status)) != cudaSuccess)
    return fail(MRI_ERR_CUDA, cudaGetErrorString(e));
  if (gemv) {
    mri::ActArgs a;
    a.xq = xq;
    a.mode = mri::ACT_I8_DEV_SCALE;
    a.scale_dev = scale;
    e = mri::launch_gemv_i8_tma(s->dev, st, static_cast<int>(m), w_dev, w_scales_dev, n, k, a, out_dev,
                                nullptr, status, nullptr);
  } else {
    e = mri::launch_gemm_i8_tc(s->dev, st, xq, scale, /*scale_per_row=*/0, w_dev, w_scales_dev, m, n, k,
                               out_dev, nullptr, status, nullptr);
  }
  return e == cudaSuccess ? MRI_OK : fail(MRI_ERR_CUDA, cudaGetErrorString(e));
}

int mri_noalloc_check_status(void* cuda_stream) {
  g_noalloc_error.clear();
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return fail(MRI_ERR_CUDA, cudaGetErrorString(e));
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  DeviceSetup* s = nullptr;
  if (int rc = setup_device(device, st, &s)) return rc;
  // The word is read through a plain copy into this stack variable after the
  // stream's work has finished, then cleared; nothing is allocated.
  int word = 0;
  int* status = reinterpret_cast<int*>(s->scratch + kStatusOffset);
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess ||
      (e = cudaMemcpyAsync(&word, status, sizeof(int), cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
      (e = cudaMemsetAsync(status, 0, sizeof(int), st)) != cudaSuccess ||
      (word != MRI_OK &&
       (e = cudaMemsetAsync(s->scratch + kSyncOffset, 0, 8, st)) != cudaSuccess) ||
      (e = cudaStreamSynchronize(st)) != cudaSuccess)
    return fail(MRI_ERR_CUDA, cudaGetErrorString(e));
  if (word != MRI_OK) {
    fail(word, "matmul_int8_from_f32_noalloc: a bounded device-side wait gave up (output incomplete)");
    return word;
  }
  return MRI_OK;
}

}  // extern "C"
