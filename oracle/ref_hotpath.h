/*
 * ref_hotpath.h — CPU ORACLE for the quantized-matmul hot path of
 * mini-rust-inference (crate `llm-inference-engine`).
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the GPU path is
 * compared against, and the timed CPU baseline of bench.py.  Nothing in the
 * product library (libmri_gpu.so) links, loads or calls it; only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs do.
 *
 * It is a plain C++ restatement of the reference's Rust functions, written so
 * that every floating-point operation happens in the same order and with the
 * same rounding as the Rust source (no FMA contraction: built with
 * -ffp-contract=off).  Each function cites the Rust file:line it follows
 * (paths relative to the reference repository root).
 *
 * Parity pinning: the reference is Rust and cannot be compiled in this
 * environment (no cargo/rustc), so the restatement is pinned against the
 * known-answer values of the reference's own unit tests, transcribed into
 * tests/golden/reference_known_answers.json by tests/golden/make_golden.py.
 *
 * Status codes mirror TensorError variants (src/tensor/error.rs:7-29):
 *   0 = Ok, 1 = InvalidShape, 2 = ShapeMismatch.
 */
#ifndef MRI_ORACLE_REF_HOTPATH_H
#define MRI_ORACLE_REF_HOTPATH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OREF_OK = 0, OREF_INVALID_SHAPE = 1, OREF_SHAPE_MISMATCH = 2 };

/* quant/int8/symmetric.rs:42-57 (and quantize_symmetric_into :63-76). */
float oref_quantize_symmetric(const float* values, size_t n, int8_t* q_out);
/* Row-wise application used by matmul_q8_0_direct (q8_direct.rs:264). */
void oref_quantize_symmetric_rows(const float* values, size_t m, size_t k,
                                  int8_t* q_out, float* scales_out);
/* quant/int8/symmetric.rs:91-93 */
void oref_dequantize_symmetric(const int8_t* q, size_t n, float scale, float* out);

/* quant/int8/per_channel.rs:98-128 */
void oref_quantize_per_channel(const float* w, size_t n_out, size_t k_in,
                               int8_t* data_out, float* scales_out);

/* ops/matmul/int8.rs:61-98.  acc_out (optional, may be NULL) receives the
 * i32 accumulators [m, n]. */
int oref_matmul_int8(const int8_t* act_q, size_t act_len, float act_scale,
                     const int8_t* w, const float* scales, size_t n_out, size_t k_in,
                     size_t m, float* out, int32_t* acc_out);

/* ops/matmul/int8.rs:113-143 (input already contiguous [m, k]). */
int oref_matmul_int8_from_f32(const float* x, size_t m, size_t k,
                              const int8_t* w, const float* scales, size_t n_out,
                              size_t k_in, float* out);

/* ops/matmul/int8_avx2.rs:136-148 (dot_i8_avx2) and :174-207 (matmul_int8_avx2). */
int32_t oref_dot_i8_avx2(const int8_t* a, const int8_t* b, size_t n);
int32_t oref_dot_i8_scalar(const int8_t* a, const int8_t* b, size_t n);
int oref_matmul_int8_avx2(const int8_t* act_q, size_t act_len, float act_scale,
                          const int8_t* w, const float* scales, size_t n_out,
                          size_t k_in, size_t m, float* out);

/* ops/matmul/parallel.rs:308-346: one task per output row m (rayon
 * par_chunks_mut(n)); n_threads <= 0 means all hardware threads.  acc_out
 * (nullable; a checker's addition) receives the i32 sums [m, n_out]. */
int oref_matmul_int8_parallel(const int8_t* act_q, size_t act_len, float act_scale,
                              const int8_t* w, const float* scales, size_t n_out,
                              size_t k_in, size_t m, float* out, int n_threads,
                              int32_t* acc_out);

/* gguf/quantization.rs:416-461 and :464-498 */
float oref_f16_to_f32(uint16_t h);
uint16_t oref_f32_to_f16(float f);

/* gguf/dequant.rs:389-424 (create_q8_0_block) and :706-749 (create_q4_0_block) */
void oref_create_q8_0_block(const float* values32, uint8_t* block34);
void oref_create_q4_0_block(const float* values32, uint8_t* block18);
/* Apply the block codec row by row to a [n_out, k_in] f32 matrix
 * (Q8_0WeightMatrix::from_f32_tensor, q8_direct.rs:118-158; q4_0 test
 * helper pack_weight, q4_0.rs:196-206).  k_in must be a multiple of 32. */
int oref_quantize_q8_0_matrix(const float* w, size_t n_out, size_t k_in, uint8_t* out);
int oref_quantize_q4_0_matrix(const float* w, size_t n_out, size_t k_in, uint8_t* out);

/* gguf/dequant.rs:103-133 and :471-500.  Return 1 (length not a multiple of
 * the block size) or 0. */
int oref_dequantize_q8_0(const uint8_t* data, size_t len, float* out);
int oref_dequantize_q4_0(const uint8_t* data, size_t len, float* out);

/* Q8_0WeightMatrix::from_raw_bytes validation (q8_direct.rs:80-107). */
int oref_q8_0_check_raw(size_t data_len, size_t n_out, size_t k_in);

/* ops/matmul/q8_direct.rs:229-289 */
int oref_matmul_q8_0_direct(const float* x, size_t m, size_t k,
                            const uint8_t* w_bytes, size_t n_out, size_t k_in,
                            float* out);

/* ops/matmul/q4_0.rs:94-181 */
int oref_matmul_q4_0_dequant(const float* x, size_t m, size_t k_x,
                             const uint8_t* w_bytes, size_t w_len,
                             size_t n_out, size_t k, float* out);

/* ── model glue around the projections (LlamaModelInt8 checker) ───────────── */
/* ops/norm/rmsnorm.rs:51-117: per row, sequential sum of squares / d,
 * rms_inv = 1 / sqrt(mean_sq + eps), out = w * (x * rms_inv). */
void oref_rmsnorm(const float* x, size_t rows, size_t d, const float* w, float eps, float* out);
/* ops/rope.rs:43-76: cos/sin tables [max_seq, head_dim/2]. */
void oref_rope_table(size_t max_seq, size_t head_dim, float base, float* cos_out, float* sin_out);
/* ops/rope.rs:121-190: x [seq, n_heads, head_dim] in place, interleaved pairs. */
void oref_rope_apply(float* x, size_t seq, size_t n_heads, size_t head_dim, const float* cos_t,
                     const float* sin_t, size_t start_pos);
/* attention/gqa.rs:217-237 + attention/sdpa.rs:168-235 + attention/mask.rs:77-115:
 * q [seq_q, n_heads*hd], k/v [seq_k, n_kv*hd] -> out [seq_q, n_heads*hd]. */
void oref_gqa_causal_offset(const float* q, const float* k, const float* v, size_t seq_q,
                            size_t seq_k, size_t n_heads, size_t n_kv_heads, size_t head_dim,
                            size_t start_pos, float* out);
/* ops/activation/swiglu.rs:39-61: silu(g) * u, silu(x) = x / (1 + exp(-x)). */
void oref_swiglu(const float* gate, const float* up, size_t n, float* out);
/* forward_int8.rs:575-580 (test helper smooth_weight), for fixtures. */
void oref_smooth_weight(size_t rows, size_t cols, float seed, float* out);

/* Hardware threads the parallel restatement would use. */
int oref_hardware_threads(void);

#ifdef __cplusplus
}
#endif
#endif
