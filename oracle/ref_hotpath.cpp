// ref_hotpath.cpp — CPU ORACLE (test infrastructure only; see ref_hotpath.h).
//
// A C++ restatement of the reference's Rust hot-path functions.  Rust float
// semantics that matter for bit-exact agreement are written out explicitly:
//   * f32::round            -> roundf (half away from zero)
//   * f32::clamp            -> NaN passes through unchanged
//   * `x as i8` / `as i32`  -> saturating cast, NaN -> 0
//   * fold(0.0, f32::max)   -> fmaxf fold from +0 (NaN operands are skipped)
//   * no FMA contraction    -> this file is compiled with -ffp-contract=off
#include "ref_hotpath.h"

#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace {

inline float rust_clamp(float x, float lo, float hi) {
  // core::f32::clamp: `if self < min { self = min } if self > max { self = max }`
  if (x < lo) x = lo;
  if (x > hi) x = hi;
  return x;
}

inline int8_t rust_as_i8(float x) {
  if (std::isnan(x)) return 0;
  if (x >= 127.0f) return 127;
  if (x <= -128.0f) return -128;
  return static_cast<int8_t>(x);  // truncation toward zero
}

inline int32_t rust_as_i32(float x) {
  if (std::isnan(x)) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return static_cast<int32_t>(x);
}

inline float abs_max_fold(const float* v, size_t n) {
  float m = 0.0f;
  for (size_t i = 0; i < n; ++i) m = std::fmax(m, std::fabs(v[i]));
  return m;
}

constexpr size_t kBlock = 32;     // QK_LEGACY, gguf/dequant.rs
constexpr size_t kQ8Bytes = 34;   // Q8_0_BLOCK_SIZE
constexpr size_t kQ4Bytes = 18;   // Q4_0_BLOCK_SIZE

}  // namespace

extern "C" {

// quant/int8/symmetric.rs:42-57
float oref_quantize_symmetric(const float* values, size_t n, int8_t* q_out) {
  const float max_abs = abs_max_fold(values, n);
  const float scale = (max_abs == 0.0f) ? 1.0f : max_abs / 127.0f;
  const float inv_scale = 1.0f / scale;
  for (size_t i = 0; i < n; ++i) {
    const float q = std::round(values[i] * inv_scale);
    q_out[i] = rust_as_i8(rust_clamp(q, -127.0f, 127.0f));
  }
  return scale;
}

// ops/matmul/q8_direct.rs:260-264 — quantize_symmetric applied per input row.
void oref_quantize_symmetric_rows(const float* values, size_t m, size_t k,
                                  int8_t* q_out, float* scales_out) {
  for (size_t r = 0; r < m; ++r)
    scales_out[r] = oref_quantize_symmetric(values + r * k, k, q_out + r * k);
}

// quant/int8/symmetric.rs:91-93
void oref_dequantize_symmetric(const int8_t* q, size_t n, float scale, float* out) {
  for (size_t i = 0; i < n; ++i) out[i] = static_cast<float>(q[i]) * scale;
}

// quant/int8/per_channel.rs:98-128
void oref_quantize_per_channel(const float* w, size_t n_out, size_t k_in,
                               int8_t* data_out, float* scales_out) {
  for (size_t n = 0; n < n_out; ++n) {
    const float* row = w + n * k_in;
    const float max_abs = abs_max_fold(row, k_in);
    const float scale = (max_abs == 0.0f) ? 1.0f : max_abs / 127.0f;
    const float inv = 1.0f / scale;
    scales_out[n] = scale;
    for (size_t k = 0; k < k_in; ++k)
      data_out[n * k_in + k] =
          rust_as_i8(rust_clamp(std::round(row[k] * inv), -127.0f, 127.0f));
  }
}

int32_t oref_dot_i8_scalar(const int8_t* a, const int8_t* b, size_t n) {
  // int8_avx2.rs dot_i8_scalar and the inner loop of int8.rs:88-91.  The
  // Rust `+=` on i32 cannot overflow for |K| < 133,000 (127*127*K < 2^31);
  // unsigned arithmetic keeps the C++ well-defined beyond that and equals
  // Rust's release-mode wrapping.
  uint32_t acc = 0;
  for (size_t i = 0; i < n; ++i)
    acc += static_cast<uint32_t>(static_cast<int32_t>(a[i]) * static_cast<int32_t>(b[i]));
  return static_cast<int32_t>(acc);
}

// ops/matmul/int8.rs:61-98
int oref_matmul_int8(const int8_t* act_q, size_t act_len, float act_scale,
                     const int8_t* w, const float* scales, size_t n_out, size_t k_in,
                     size_t m, float* out, int32_t* acc_out) {
  if (act_len != m * k_in) return OREF_INVALID_SHAPE;
  for (size_t mi = 0; mi < m; ++mi) {
    const int8_t* a_row = act_q + mi * k_in;
    for (size_t ni = 0; ni < n_out; ++ni) {
      const int32_t acc = oref_dot_i8_scalar(a_row, w + ni * k_in, k_in);
      if (acc_out) acc_out[mi * n_out + ni] = acc;
      // `acc as f32 * act_scale * weights.scales[n_i]`, left to right.
      out[mi * n_out + ni] = (static_cast<float>(acc) * act_scale) * scales[ni];
    }
  }
  return OREF_OK;
}

// ops/matmul/int8.rs:113-143
int oref_matmul_int8_from_f32(const float* x, size_t m, size_t k,
                              const int8_t* w, const float* scales, size_t n_out,
                              size_t k_in, float* out) {
  if (k != k_in) return OREF_SHAPE_MISMATCH;
  std::vector<int8_t> act_q(m * k);
  const float s = oref_quantize_symmetric(x, m * k, act_q.data());
  return oref_matmul_int8(act_q.data(), act_q.size(), s, w, scales, n_out, k_in, m,
                          out, nullptr);
}

#if defined(__x86_64__)
// ops/matmul/int8_avx2.rs:49-60 (horizontal add of eight i32 lanes)
__attribute__((target("avx2"))) static int32_t hsum_epi32_avx2(__m256i v) {
  __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
  return _mm_cvtsi128_si32(s);
}

// ops/matmul/int8_avx2.rs:69-111.  32 bytes per step: |a| (as u8) times b
// with a's sign applied (vpmaddubsw), widened pairwise to i32 (vpmaddwd),
// then a scalar tail.  Like the reference it is exact only while no byte of
// `a` is -128 (the reference's activations are clamped to [-127, 127]).
__attribute__((target("avx2"))) static int32_t dot_i8_avx2_impl(const int8_t* a,
                                                                const int8_t* b,
                                                                size_t n) {
  const size_t chunks = n / 32;
  const __m256i ones = _mm256_set1_epi16(1);
  __m256i acc = _mm256_setzero_si256();
  for (size_t i = 0; i < chunks; ++i) {
    const __m256i va = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(a + i * 32));
    const __m256i vb = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(b + i * 32));
    const __m256i pairs = _mm256_maddubs_epi16(_mm256_abs_epi8(va), _mm256_sign_epi8(vb, va));
    acc = _mm256_add_epi32(acc, _mm256_madd_epi16(pairs, ones));
  }
  int32_t result = hsum_epi32_avx2(acc);
  for (size_t i = chunks * 32; i < n; ++i)
    result += static_cast<int32_t>(a[i]) * static_cast<int32_t>(b[i]);
  return result;
}
#endif

// ops/matmul/int8_avx2.rs:136-148 (runtime feature check, scalar fallback)
int32_t oref_dot_i8_avx2(const int8_t* a, const int8_t* b, size_t n) {
#if defined(__x86_64__)
  if (__builtin_cpu_supports("avx2")) return dot_i8_avx2_impl(a, b, n);
#endif
  return oref_dot_i8_scalar(a, b, n);
}

// ops/matmul/int8_avx2.rs:174-207
int oref_matmul_int8_avx2(const int8_t* act_q, size_t act_len, float act_scale,
                          const int8_t* w, const float* scales, size_t n_out,
                          size_t k_in, size_t m, float* out) {
  if (act_len != m * k_in) return OREF_INVALID_SHAPE;
  for (size_t mi = 0; mi < m; ++mi)
    for (size_t ni = 0; ni < n_out; ++ni) {
      const int32_t acc = oref_dot_i8_avx2(act_q + mi * k_in, w + ni * k_in, k_in);
      out[mi * n_out + ni] = (static_cast<float>(acc) * act_scale) * scales[ni];
    }
  return OREF_OK;
}

int oref_hardware_threads(void) {
  const unsigned t = std::thread::hardware_concurrency();
  return t == 0 ? 1 : static_cast<int>(t);
}

// ops/matmul/parallel.rs:308-346.  rayon's par_chunks_mut(n) hands out one
// output row per task; here a fixed pool pulls row indices from an atomic
// counter.  At m == 1 exactly one thread works, as in the reference.
// acc_out (nullable, not in the reference's signature) receives the i32 dot
// of every (row, column) before the epilogue, for checks of INT32 sums.
int oref_matmul_int8_parallel(const int8_t* act_q, size_t act_len, float act_scale,
                              const int8_t* w, const float* scales, size_t n_out,
                              size_t k_in, size_t m, float* out, int n_threads,
                              int32_t* acc_out) {
  if (act_len != m * k_in) return OREF_INVALID_SHAPE;
  size_t threads = n_threads > 0 ? static_cast<size_t>(n_threads)
                                 : static_cast<size_t>(oref_hardware_threads());
  if (threads > m) threads = m;
  if (threads == 0) return OREF_OK;
  std::atomic<size_t> next{0};
  auto worker = [&]() {
    for (;;) {
      const size_t mi = next.fetch_add(1);
      if (mi >= m) break;
      const int8_t* a_row = act_q + mi * k_in;
      float* out_row = out + mi * n_out;
      for (size_t ni = 0; ni < n_out; ++ni) {
        const int32_t acc = oref_dot_i8_avx2(a_row, w + ni * k_in, k_in);
        if (acc_out) acc_out[mi * n_out + ni] = acc;
        out_row[ni] = (static_cast<float>(acc) * act_scale) * scales[ni];
      }
    }
  };
  if (threads == 1) {
    worker();
    return OREF_OK;
  }
  std::vector<std::thread> pool;
  pool.reserve(threads - 1);
  for (size_t t = 1; t < threads; ++t) pool.emplace_back(worker);
  worker();
  for (auto& th : pool) th.join();
  return OREF_OK;
}

// gguf/quantization.rs:416-461
float oref_f16_to_f32(uint16_t h) {
  const unsigned sign = (h >> 15) & 1u;
  const unsigned exp = (h >> 10) & 0x1Fu;
  const unsigned mant = h & 0x3FFu;
  if (exp == 0) {
    if (mant == 0) return sign ? -0.0f : 0.0f;
    const float val = (static_cast<float>(mant) * (1.0f / 1024.0f)) * (1.0f / 16384.0f);
    return sign ? -val : val;
  }
  if (exp == 31) {
    if (mant == 0) return sign ? -INFINITY : INFINITY;
    return NAN;
  }
  // (1 + mant/1024) * 2^(exp-15); powi(2, e) is an exact power of two here.
  const float val = (1.0f + static_cast<float>(mant) / 1024.0f) *
                    std::ldexp(1.0f, static_cast<int>(exp) - 15);
  return sign ? -val : val;
}

// gguf/quantization.rs:464-498.  Truncating conversion, restated exactly,
// including its subnormal branch (shift by 126-exp+13).
uint16_t oref_f32_to_f16(float f) {
  uint32_t bits;
  std::memcpy(&bits, &f, 4);
  const uint16_t sign = static_cast<uint16_t>((bits >> 31) & 1u);
  const int32_t exp = static_cast<int32_t>((bits >> 23) & 0xFFu);
  const uint32_t mant = bits & 0x7FFFFFu;
  if (exp == 255) {
    if (mant == 0) return static_cast<uint16_t>((sign << 15) | 0x7C00u);
    uint16_t m16 = static_cast<uint16_t>(mant >> 13);
    if (m16 < 1) m16 = 1;
    return static_cast<uint16_t>((sign << 15) | 0x7C00u | m16);
  }
  if (exp > 142) return static_cast<uint16_t>((sign << 15) | 0x7C00u);
  if (exp < 103) return static_cast<uint16_t>(sign << 15);
  if (exp < 113) {
    const uint32_t mant_with_implicit = mant | 0x800000u;
    const int32_t shift = 126 - exp;
    const uint16_t mant16 = static_cast<uint16_t>(mant_with_implicit >> (shift + 13));
    return static_cast<uint16_t>((sign << 15) | mant16);
  }
  const uint16_t exp16 = static_cast<uint16_t>((exp - 112) & 0x1F);
  const uint16_t mant16 = static_cast<uint16_t>(mant >> 13);
  return static_cast<uint16_t>((sign << 15) | (exp16 << 10) | mant16);
}

// gguf/dequant.rs:389-424
void oref_create_q8_0_block(const float* values, uint8_t* block) {
  const float max_abs = abs_max_fold(values, kBlock);
  const float scale = (max_abs == 0.0f) ? 0.0f : max_abs / 127.0f;
  const uint16_t h = oref_f32_to_f16(scale);
  std::memset(block, 0, kQ8Bytes);
  block[0] = static_cast<uint8_t>(h & 0xFF);
  block[1] = static_cast<uint8_t>(h >> 8);
  if (scale > 0.0f) {
    const float inv_scale = 1.0f / scale;  // the f32 scale, not the f16 one
    for (size_t i = 0; i < kBlock; ++i) {
      const int8_t q = rust_as_i8(rust_clamp(std::round(values[i] * inv_scale), -128.0f, 127.0f));
      block[2 + i] = static_cast<uint8_t>(q);
    }
  }
}

// gguf/dequant.rs:706-749
void oref_create_q4_0_block(const float* values, uint8_t* block) {
  const float max_abs = abs_max_fold(values, kBlock);
  const float scale = (max_abs == 0.0f) ? 0.0f : max_abs / 7.0f;
  const uint16_t h = oref_f32_to_f16(scale);
  std::memset(block, 0, kQ4Bytes);
  block[0] = static_cast<uint8_t>(h & 0xFF);
  block[1] = static_cast<uint8_t>(h >> 8);
  if (scale > 0.0f) {
    const float inv_scale = 1.0f / scale;
    for (size_t i = 0; i < 16; ++i) {
      auto nib = [&](float v) -> uint8_t {
        int64_t q = static_cast<int64_t>(rust_as_i32(std::round(v * inv_scale))) + 8;
        if (q < 0) q = 0;
        if (q > 15) q = 15;
        return static_cast<uint8_t>(q);
      };
      block[2 + i] = static_cast<uint8_t>(nib(values[2 * i]) | (nib(values[2 * i + 1]) << 4));
    }
  } else {
    for (size_t i = 0; i < 16; ++i) block[2 + i] = 0x88;
  }
}

// q8_direct.rs:118-158 (row-major blocks, 34 bytes each)
int oref_quantize_q8_0_matrix(const float* w, size_t n_out, size_t k_in, uint8_t* out) {
  if (k_in % kBlock != 0) return OREF_INVALID_SHAPE;
  const size_t nb = k_in / kBlock;
  for (size_t r = 0; r < n_out; ++r)
    for (size_t b = 0; b < nb; ++b)
      oref_create_q8_0_block(w + r * k_in + b * kBlock, out + (r * nb + b) * kQ8Bytes);
  return OREF_OK;
}

// q4_0.rs:196-206 (pack_weight: rows of 18-byte blocks)
int oref_quantize_q4_0_matrix(const float* w, size_t n_out, size_t k_in, uint8_t* out) {
  if (k_in % kBlock != 0) return OREF_INVALID_SHAPE;
  const size_t nb = k_in / kBlock;
  for (size_t r = 0; r < n_out; ++r)
    for (size_t b = 0; b < nb; ++b)
      oref_create_q4_0_block(w + r * k_in + b * kBlock, out + (r * nb + b) * kQ4Bytes);
  return OREF_OK;
}

static inline float block_d(const uint8_t* blk) {
  return oref_f16_to_f32(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
}

// gguf/dequant.rs:103-133
int oref_dequantize_q8_0(const uint8_t* data, size_t len, float* out) {
  if (len % kQ8Bytes != 0) return 1;
  const size_t nb = len / kQ8Bytes;
  for (size_t b = 0; b < nb; ++b) {
    const uint8_t* blk = data + b * kQ8Bytes;
    const float scale = block_d(blk);
    for (size_t i = 0; i < kBlock; ++i)
      out[b * kBlock + i] = scale * static_cast<float>(static_cast<int8_t>(blk[2 + i]));
  }
  return 0;
}

// gguf/dequant.rs:471-500
int oref_dequantize_q4_0(const uint8_t* data, size_t len, float* out) {
  if (len % kQ4Bytes != 0) return 1;
  const size_t nb = len / kQ4Bytes;
  for (size_t b = 0; b < nb; ++b) {
    const uint8_t* blk = data + b * kQ4Bytes;
    const float scale = block_d(blk);
    for (size_t i = 0; i < 16; ++i) {
      const uint8_t byte = blk[2 + i];
      out[b * kBlock + 2 * i] = scale * static_cast<float>(static_cast<int>(byte & 0x0F) - 8);
      out[b * kBlock + 2 * i + 1] = scale * static_cast<float>(static_cast<int>((byte >> 4) & 0x0F) - 8);
    }
  }
  return 0;
}

// q8_direct.rs:80-107
int oref_q8_0_check_raw(size_t data_len, size_t n_out, size_t k_in) {
  if (k_in % kBlock != 0) return OREF_INVALID_SHAPE;
  if (data_len != n_out * (k_in / kBlock) * kQ8Bytes) return OREF_INVALID_SHAPE;
  return OREF_OK;
}

// ops/matmul/q8_direct.rs:229-289.  Per row: quantize_symmetric(row); per
// (m, n): acc += dot_i32(block) as f32 * s_a * d(n, b), blocks in order.
int oref_matmul_q8_0_direct(const float* x, size_t m, size_t k,
                            const uint8_t* w_bytes, size_t n_out, size_t k_in,
                            float* out) {
  if (k != k_in) return OREF_SHAPE_MISMATCH;
  const size_t nb = k_in / kBlock;
  std::vector<int8_t> act_q(k);
  for (size_t mi = 0; mi < m; ++mi) {
    const float s_a = oref_quantize_symmetric(x + mi * k, k, act_q.data());
    for (size_t ni = 0; ni < n_out; ++ni) {
      float acc = 0.0f;
      for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = w_bytes + (ni * nb + b) * kQ8Bytes;
        const float w_scale = block_d(blk);
        int32_t dot = 0;
        for (size_t i = 0; i < kBlock; ++i)
          dot += static_cast<int32_t>(act_q[b * kBlock + i]) *
                 static_cast<int32_t>(static_cast<int8_t>(blk[2 + i]));
        acc += (static_cast<float>(dot) * s_a) * w_scale;
      }
      out[mi * n_out + ni] = acc;
    }
  }
  return OREF_OK;
}

// ops/matmul/q4_0.rs:94-181.  Validation order follows the source: K
// mismatch, then k % 32, then byte length.
int oref_matmul_q4_0_dequant(const float* x, size_t m, size_t k_x,
                             const uint8_t* w_bytes, size_t w_len,
                             size_t n_out, size_t k, float* out) {
  if (k_x != k) return OREF_SHAPE_MISMATCH;
  if (k % kBlock != 0) return OREF_INVALID_SHAPE;
  const size_t nb = k / kBlock;
  if (w_len != n_out * nb * kQ4Bytes) return OREF_INVALID_SHAPE;
  float buf[kBlock];
  for (size_t n = 0; n < n_out; ++n) {
    const uint8_t* row = w_bytes + n * nb * kQ4Bytes;
    for (size_t mi = 0; mi < m; ++mi) {
      float acc = 0.0f;
      const float* inp = x + mi * k;
      for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * kQ4Bytes;
        const float scale = block_d(blk);  // dequant_block_into, q4_0.rs:59-68
        for (size_t i = 0; i < 16; ++i) {
          const uint8_t byte = blk[2 + i];
          buf[2 * i] = scale * static_cast<float>(static_cast<int>(byte & 0x0F) - 8);
          buf[2 * i + 1] = scale * static_cast<float>(static_cast<int>((byte >> 4) & 0x0F) - 8);
        }
        for (size_t i = 0; i < kBlock; ++i) acc += inp[b * kBlock + i] * buf[i];
      }
      out[mi * n_out + n] = acc;
    }
  }
  return OREF_OK;
}

// ── model glue ──────────────────────────────────────────────────────────────

// ops/norm/rmsnorm.rs:51-117
void oref_rmsnorm(const float* x, size_t rows, size_t d, const float* w, float eps, float* out) {
  for (size_t r = 0; r < rows; ++r) {
    const float* xr = x + r * d;
    float sum = 0.0f;
    for (size_t i = 0; i < d; ++i) sum += xr[i] * xr[i];
    const float mean_sq = sum / static_cast<float>(d);
    const float rms_inv = 1.0f / std::sqrt(mean_sq + eps);
    for (size_t i = 0; i < d; ++i) out[r * d + i] = w[i] * (xr[i] * rms_inv);
  }
}

// ops/rope.rs:43-76
void oref_rope_table(size_t max_seq, size_t head_dim, float base, float* cos_out, float* sin_out) {
  const size_t half = head_dim / 2;
  std::vector<float> thetas(half);
  for (size_t i = 0; i < half; ++i)
    thetas[i] = 1.0f / std::pow(base, 2.0f * static_cast<float>(i) / static_cast<float>(head_dim));
  for (size_t pos = 0; pos < max_seq; ++pos)
    for (size_t i = 0; i < half; ++i) {
      const float angle = static_cast<float>(pos) * thetas[i];
      cos_out[pos * half + i] = std::cos(angle);
      sin_out[pos * half + i] = std::sin(angle);
    }
}

// ops/rope.rs:121-190
void oref_rope_apply(float* x, size_t seq, size_t n_heads, size_t head_dim, const float* cos_t,
                     const float* sin_t, size_t start_pos) {
  const size_t half = head_dim / 2;
  for (size_t s = 0; s < seq; ++s) {
    const size_t pos = start_pos + s;
    for (size_t h = 0; h < n_heads; ++h) {
      float* base = x + s * n_heads * head_dim + h * head_dim;
      for (size_t i = 0; i < half; ++i) {
        const float c = cos_t[pos * half + i], sn = sin_t[pos * half + i];
        const float x0 = base[2 * i], x1 = base[2 * i + 1];
        base[2 * i] = x0 * c - x1 * sn;
        base[2 * i + 1] = x1 * c + x0 * sn;
      }
    }
  }
}

// ops/softmax.rs:36-57
static void softmax_row(float* row, size_t n) {
  if (n == 0) return;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, row[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    row[i] = std::exp(row[i] - mx);
    sum += row[i];
  }
  const float inv_sum = 1.0f / sum;
  for (size_t i = 0; i < n; ++i) row[i] *= inv_sum;
}

// attention/gqa.rs:217-237, attention/sdpa.rs:168-235, attention/mask.rs:77-115
void oref_gqa_causal_offset(const float* q, const float* k, const float* v, size_t seq_q,
                            size_t seq_k, size_t n_heads, size_t n_kv_heads, size_t head_dim,
                            size_t start_pos, float* out) {
  const size_t groups = n_heads / n_kv_heads;
  const size_t qd = n_heads * head_dim, kvd = n_kv_heads * head_dim;
  const float scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
  std::vector<float> scores(seq_q * seq_k), acc(seq_q * head_dim);
  for (size_t h = 0; h < n_heads; ++h) {
    const size_t kv_h = h / groups;
    // scores = q_h @ k_h^T in the ikj order of matmul_naive (sequential over p)
    std::fill(scores.begin(), scores.end(), 0.0f);
    for (size_t i = 0; i < seq_q; ++i)
      for (size_t p = 0; p < head_dim; ++p) {
        const float a = q[i * qd + h * head_dim + p];
        for (size_t j = 0; j < seq_k; ++j) scores[i * seq_k + j] += a * k[j * kvd + kv_h * head_dim + p];
      }
    for (size_t i = 0; i < seq_q; ++i) {
      const size_t abs_pos = start_pos + i;
      for (size_t j = 0; j < seq_k; ++j) {
        const float bias = j > abs_pos ? -INFINITY : 0.0f;
        scores[i * seq_k + j] = scores[i * seq_k + j] * scale + bias;
      }
      softmax_row(&scores[i * seq_k], seq_k);
    }
    std::fill(acc.begin(), acc.end(), 0.0f);
    for (size_t i = 0; i < seq_q; ++i)
      for (size_t p = 0; p < seq_k; ++p) {
        const float wgt = scores[i * seq_k + p];
        for (size_t j = 0; j < head_dim; ++j) acc[i * head_dim + j] += wgt * v[p * kvd + kv_h * head_dim + j];
      }
    for (size_t i = 0; i < seq_q; ++i)
      for (size_t j = 0; j < head_dim; ++j) out[i * qd + h * head_dim + j] = acc[i * head_dim + j];
  }
}

// ops/activation/swiglu.rs:39-61, silu.rs:23-26
void oref_swiglu(const float* gate, const float* up, size_t n, float* out) {
  for (size_t i = 0; i < n; ++i) {
    const float g = gate[i];
    out[i] = (g / (1.0f + std::exp(-g))) * up[i];
  }
}

// model/llama/forward_int8.rs:575-580
void oref_smooth_weight(size_t rows, size_t cols, float seed, float* out) {
  const float total = static_cast<float>(rows * cols);
  for (size_t i = 0; i < rows * cols; ++i)
    out[i] = std::sin(static_cast<float>(i) * seed * 0.01f - total * seed * 0.005f) * 0.5f;
}

}  // extern "C"
