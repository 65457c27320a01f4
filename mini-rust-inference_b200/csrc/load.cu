// load.cu — GGUF tensor data straight to device weights.
//
// LlamaModelInt8::from_loader (src/model/llama/forward_int8.rs:461-507) reads
// every tensor through TensorExtractor::extract (src/gguf/extract.rs:719-737),
// which dequantizes F32 / F16 / Q8_0 / Q4_0 storage to an f32 host tensor
// (dequantize_q8_0 / dequantize_q4_0, src/gguf/dequant.rs:103-133, 471-506;
// f16_to_f32, src/gguf/quantization.rs:416-461), and then requantizes each
// projection per output row (quantize_tensor, forward_int8.rs:52-62 ->
// quantize_per_channel, src/quant/int8/per_channel.rs:98-128).
//
// Here the raw GGUF bytes cross PCIe once and both steps run on the device in
// one kernel: one CTA per output row makes two passes over the row's source
// bytes (absmax of the dequantized values, then the quantization), so no f32
// copy of the tensor exists anywhere.  Every dequantized value is exact in f32
// (an f16 scale times an integer of at most 8 bits), the absmax is
// order-independent and the quantization uses the reference's IEEE steps, so
// the INT8 rows and scales are bit-identical to the host path.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace mri {
namespace {

constexpr int kLoadThreads = 256;
// Source bytes moved to the device per conversion step.
constexpr size_t kLoadChunkBytes = size_t(256) << 20;

// Element i of a GGUF tensor stored as type T, as extract() yields it.
template <int T>
__device__ __forceinline__ float gguf_value(const uint8_t* __restrict__ src, size_t i) {
  if constexpr (T == MRI_GGML_F32) {
    return reinterpret_cast<const float*>(src)[i];
  } else if constexpr (T == MRI_GGML_F16) {
    return f16_bits_to_f32(reinterpret_cast<const uint16_t*>(src)[i]);
  } else if constexpr (T == MRI_GGML_Q8_0) {
    // dequant.rs:118-129: [f16 d LE][32 x i8], value = d * q.
    const uint8_t* b = src + (i >> 5) * 34;
    const float d = f16_bits_to_f32(b[0] | (uint32_t(b[1]) << 8));
    return __fmul_rn(d, static_cast<float>(static_cast<int8_t>(b[2 + (i & 31)])));
  } else {
    // dequant.rs:484-502: [f16 d LE][16 bytes]; byte j holds element 2j in
    // its low nibble and 2j+1 in its high nibble, value = d * (nibble - 8).
    const uint8_t* b = src + (i >> 5) * 18;
    const float d = f16_bits_to_f32(b[0] | (uint32_t(b[1]) << 8));
    const uint32_t j = static_cast<uint32_t>(i & 31);
    const uint32_t byte = b[2 + (j >> 1)];
    const int q = static_cast<int>((j & 1) ? (byte >> 4) : (byte & 15u)) - 8;
    return __fmul_rn(d, static_cast<float>(q));
  }
}

// quantize_per_channel of the dequantized rows: row r of the chunk -> q +
// r * q_stride, its scale -> scales[r * s_stride].
template <int T>
__global__ void __launch_bounds__(kLoadThreads)
    gguf_requant_rows_kernel(const uint8_t* __restrict__ src, size_t cols,
                             int8_t* __restrict__ q, size_t q_stride,
                             float* __restrict__ scales, size_t s_stride) {
  __shared__ float warp_amax[kLoadThreads / 32];
  const size_t row = blockIdx.x;
  const size_t base = row * cols;
  float m = 0.0f;
  for (size_t j = threadIdx.x; j < cols; j += kLoadThreads)
    m = absmax_acc(m, gguf_value<T>(src, base + j));
  m = warp_max(m);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_amax[warp] = m;
  __syncthreads();
  float amax = 0.0f;
#pragma unroll
  for (int w = 0; w < kLoadThreads / 32; ++w) amax = fmaxf(amax, warp_amax[w]);
  // per_channel.rs:113-115
  const float scale = sym_scale(amax);
  const float inv = __fdiv_rn(1.0f, scale);
  int8_t* out = q + row * q_stride;
  for (size_t j = threadIdx.x; j < cols; j += kLoadThreads)
    out[j] = sym_quant(gguf_value<T>(src, base + j), inv);
  if (threadIdx.x == 0) scales[row * s_stride] = scale;
}

template <int T>
__global__ void __launch_bounds__(kLoadThreads)
    gguf_dequant_kernel(const uint8_t* __restrict__ src, size_t n, float* __restrict__ out) {
  for (size_t i = blockIdx.x * size_t(kLoadThreads) + threadIdx.x; i < n;
       i += size_t(gridDim.x) * kLoadThreads)
    out[i] = gguf_value<T>(src, i);
}

template <int T>
void launch_convert(cudaStream_t st, const uint8_t* src, size_t rows, size_t cols,
                    const GgufDst& d, size_t row0) {
  if (d.f32) {
    const size_t n = rows * cols;
    const unsigned grid = static_cast<unsigned>(std::min<size_t>((n + kLoadThreads - 1) / kLoadThreads, 148 * 16));
    gguf_dequant_kernel<T><<<grid, kLoadThreads, 0, st>>>(src, n, d.f32 + row0 * cols);
  } else {
    gguf_requant_rows_kernel<T><<<static_cast<unsigned>(rows), kLoadThreads, 0, st>>>(
        src, cols, d.q + row0 * d.q_stride, d.q_stride, d.scales + row0 * d.s_stride, d.s_stride);
  }
}

}  // namespace

size_t gguf_type_bytes(int type, size_t numel) {
  switch (type) {
    case MRI_GGML_F32: return numel * 4;
    case MRI_GGML_F16: return numel * 2;
    case MRI_GGML_Q8_0: return numel / 32 * 34;
    case MRI_GGML_Q4_0: return numel / 32 * 18;
    default: return 0;
  }
}

int gguf_check(int type, size_t len, size_t numel, std::string* err) {
  char buf[200];
  const bool block = type == MRI_GGML_Q8_0 || type == MRI_GGML_Q4_0;
  if (type != MRI_GGML_F32 && type != MRI_GGML_F16 && !block) {
    // extract.rs:733-736 (GgufError::TypeMismatch)
    snprintf(buf, sizeof(buf), "type mismatch: expected F32, F16, Q8_0, or Q4_0, got ggml type %d",
             type);
    *err = buf;
    return MRI_ERR_INVALID_ARGUMENT;
  }
  if (block && numel % 32 != 0) {
    // extract.rs:458-463 / 615-620
    snprintf(buf, sizeof(buf), "shape mismatch: expected %zu elements, got %zu",
             numel - numel % 32 + 32, numel);
    *err = buf;
    return MRI_ERR_SHAPE_MISMATCH;
  }
  const size_t expected = gguf_type_bytes(type, numel);
  if (len != expected) {
    // extract.rs:171-176 / 468-473 / 625-630
    snprintf(buf, sizeof(buf), "shape mismatch: expected %zu bytes, got %zu", expected, len);
    *err = buf;
    return MRI_ERR_SHAPE_MISMATCH;
  }
  return MRI_OK;
}

int gguf_to_device(cudaStream_t st, int type, const uint8_t* bytes, size_t len, size_t rows,
                   size_t cols, const GgufDst& d, std::string* err) {
  const size_t numel = rows * cols;
  if (int rc = gguf_check(type, len, numel, err)) return rc;
  // quantize_per_channel gives each row of an empty-width matrix scale 1.
  if (rows == 0 || (cols == 0 && d.f32)) return MRI_OK;
  if (!bytes && len) {
    *err = "null tensor data";
    return MRI_ERR_INVALID_ARGUMENT;
  }
  // Whole rows per step.  A block format whose rows do not end on a block
  // boundary has blocks that straddle rows: it goes in one step.
  const bool block = type == MRI_GGML_Q8_0 || type == MRI_GGML_Q4_0;
  const size_t row_bytes = gguf_type_bytes(type, cols);
  size_t step_rows = rows;
  if (!(block && cols % 32 != 0))
    step_rows = std::max<size_t>(1, std::min(rows, kLoadChunkBytes / std::max<size_t>(row_bytes, 1)));
  const size_t step_bytes = block && cols % 32 != 0 ? len : step_rows * row_bytes;
  uint8_t* buf = nullptr;
  cudaError_t e = cudaMalloc(&buf, step_bytes + 16);
  if (e != cudaSuccess) {
    *err = std::string("cudaMalloc: ") + cudaGetErrorString(e);
    return MRI_ERR_CUDA;
  }
  for (size_t r0 = 0; r0 < rows && e == cudaSuccess; r0 += step_rows) {
    const size_t nr = std::min(step_rows, rows - r0);
    const size_t off = block && cols % 32 != 0 ? 0 : r0 * row_bytes;
    const size_t nb = block && cols % 32 != 0 ? len : nr * row_bytes;
    if (nb) e = cudaMemcpyAsync(buf, bytes + off, nb, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) break;
    switch (type) {
      case MRI_GGML_F32: launch_convert<MRI_GGML_F32>(st, buf, nr, cols, d, r0); break;
      case MRI_GGML_F16: launch_convert<MRI_GGML_F16>(st, buf, nr, cols, d, r0); break;
      case MRI_GGML_Q8_0: launch_convert<MRI_GGML_Q8_0>(st, buf, nr, cols, d, r0); break;
      default: launch_convert<MRI_GGML_Q4_0>(st, buf, nr, cols, d, r0); break;
    }
    e = cudaGetLastError();
    // The next step overwrites the staging buffer.
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  cudaFree(buf);
  if (e != cudaSuccess) {
    *err = std::string("GGUF tensor conversion: ") + cudaGetErrorString(e);
    return MRI_ERR_CUDA;
  }
  return MRI_OK;
}

}  // namespace mri
