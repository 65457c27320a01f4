/*
 * mri_gpu.h — C ABI of the B200 (sm_100a) quantized-matmul hot path of
 * mini-rust-inference.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, and
 * returns an int32 status.  The reference's operators are Rust free functions
 * returning Result<Tensor<f32>, TensorError>; the status codes map 1:1 onto
 * that error enum (src/tensor/error.rs:7-29):
 *   MRI_ERR_INVALID_SHAPE  <-> TensorError::InvalidShape
 *   MRI_ERR_SHAPE_MISMATCH <-> TensorError::ShapeMismatch
 * and mri_last_error() returns the reason text of the calling thread's last
 * failure (the `reason` / expected-vs-got of the Rust error).
 *
 * Conventions
 *   - Weights live on the device: QuantizedMatrix, Q8_0WeightMatrix and the
 *     Q4_0 byte slice are uploaded once into opaque handles (the reference
 *     loads them once in LlamaModelInt8::from_loader, forward_int8.rs:461-507).
 *   - `*_dev` pointers are device memory; calls on them are asynchronous on
 *     the context's stream.  `mri_host_*` calls take host memory and are
 *     synchronous (H2D, kernels, D2H, stream sync) — they are the drop-ins for
 *     the reference functions, which take and return host tensors.
 *   - A context owns one CUDA stream and its scratch buffers; use one context
 *     per host thread (the reference functions are reentrant; contexts give the
 *     same property).
 *   - There is no CPU fallback: without a usable sm_100 device every compute
 *     call returns MRI_ERR_CUDA.
 */
#ifndef MRI_GPU_H
#define MRI_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MRI_ABI_VERSION 1

#if defined(__GNUC__)
#define MRI_API __attribute__((visibility("default")))
#else
#define MRI_API
#endif

enum mri_status {
  MRI_OK = 0,
  MRI_ERR_INVALID_SHAPE = 1,   /* TensorError::InvalidShape */
  MRI_ERR_SHAPE_MISMATCH = 2,  /* TensorError::ShapeMismatch */
  MRI_ERR_CUDA = 3,            /* CUDA runtime / driver failure, no device */
  MRI_ERR_COMM = 4,            /* NCCL failure (sharded calls) */
  MRI_ERR_TIMEOUT = 5,         /* a bounded device-side wait gave up */
  MRI_ERR_INVALID_ARGUMENT = 6 /* null handle or pointer, bad enum value */
};

/* Activation-quantization granularity. */
enum mri_granularity {
  MRI_PER_TENSOR = 0, /* one scale for all M*K values: quantize_symmetric over
                         the whole [M,K] buffer (int8.rs:141, forward_int8.rs:94) */
  MRI_PER_ROW = 1     /* one scale per row (q8_direct.rs:260-264) */
};

typedef struct mri_ctx mri_ctx;
typedef struct mri_qmatrix mri_qmatrix;         /* QuantizedMatrix, per_channel.rs:29-40 */
typedef struct mri_q8_0_matrix mri_q8_0_matrix; /* Q8_0WeightMatrix, q8_direct.rs:60-69 */
typedef struct mri_q4_0_matrix mri_q4_0_matrix; /* Q4_0 bytes + (n_out, k), q4_0.rs:94-99 */

MRI_API int mri_abi_version(void);
/* Reason text of the calling thread's last failed call ("" if none). */
MRI_API const char* mri_last_error(void);

/* ── context ──────────────────────────────────────────────────────────────── */
/* Creates a context on `device` with its own non-blocking stream. */
MRI_API int mri_ctx_create(int device, mri_ctx** out);
/* Same, but enqueues on the caller's `cudaStream_t` (not owned). */
MRI_API int mri_ctx_create_on_stream(int device, void* cuda_stream, mri_ctx** out);
MRI_API int mri_ctx_destroy(mri_ctx* ctx);
MRI_API int mri_ctx_synchronize(mri_ctx* ctx);
MRI_API void* mri_ctx_stream(mri_ctx* ctx);
/* Reads and clears the device-side status word that bounded waits write
 * (MRI_OK or MRI_ERR_TIMEOUT).  Synchronizes the stream. */
MRI_API int mri_ctx_check_device_status(mri_ctx* ctx);
/* Number of kernels this context has launched (for launch accounting). */
MRI_API uint64_t mri_ctx_launch_count(const mri_ctx* ctx);

/* Kernel-variant options of a context.  No counterpart in the reference (its
 * kernel choice is fixed at build time, src/ops/matmul/parallel.rs:258-275).
 * The defaults are the measured best choices; every other value selects a
 * variant that computes the same result (bit for bit where the product is
 * bit-exact) and exists for tests and measurements.  Options apply to
 * launches made after the call; a model's decode graph keeps the variant it
 * was captured with.  In a sharded job every rank sets the same values.
 * Unknown option or value out of range -> MRI_ERR_INVALID_ARGUMENT. */
enum mri_option {
  MRI_OPT_PDL = 0,        /* 1 (default): programmatic dependent launch between kernels; 0: off */
  MRI_OPT_GEMM_BN = 1,    /* 0 (default): GEMM tile width per shape; 128..256 (step 32): forced */
  MRI_OPT_GEMM_2CTA = 2,  /* 1 (default): between one and two rounds of GEMM tiles, one tile per CTA
                             and two CTAs per SM; 0: the persistent grid */
  MRI_OPT_Q8_MMA = 3,     /* 1 (default): Q8_0 at m = 2..8 on the integer warp MMA; 0: streaming kernel */
  MRI_OPT_Q4_MMA = 4,     /* 1 (default): Q4_0 at m = 2..8 on the bf16 warp MMA; 0: streaming kernel */
  MRI_OPT_TC_ATTN = 5,    /* 1 (default): tensor-core prefill attention for head dim 64 / 128;
                             0: the CUDA-core kernel */
  MRI_OPT_FA_SPLIT = 6,   /* 3 (default): prefill key walks of at least this many 64-key tiles are
                             split over two blocks; 0: never */
  MRI_OPT_SHARD_PEER = 7  /* sharded products: 2 (default) gathered over peer memory for m > 8 (the
                             GEMM epilogue writes each tile to every rank) and by NCCL for m <= 8;
                             1: over peer memory for every m; 0: NCCL for every m */,
  MRI_OPT_GEMM_PAIR = 8   /* 1 (default): tensor-core GEMMs with a plain output (no residual, no
                             INT32 copy) run on CTA pairs (tcgen05.mma.cta_group::2, 256-row tiles)
                             from four rounds of pair tiles on; 2: pairs for any plain output of
                             more than 128 rows; 0: one CTA per tile */,
  MRI_OPT_Q4_LIMB = 9     /* 1 (default): Q4_0 at m = 1 with K % 1024 == 0 on exact integer block
                             dots (21-bit activation digits, dp4a); 0: the f32 streaming kernel */
};
MRI_API int mri_ctx_set_option(mri_ctx* ctx, int option, int value);
MRI_API int mri_ctx_get_option(mri_ctx* ctx, int option, int* value);

/* ── device-resident weights ──────────────────────────────────────────────── */
/* QuantizedMatrix { data: [n_out,k_in] i8 row-major, scales: [n_out] f32 }
 * (per_channel.rs:29-40).  Host pointers; synchronous upload. */
MRI_API int mri_qmatrix_upload(mri_ctx* ctx, const int8_t* data, const float* scales,
                       size_t n_out, size_t k_in, mri_qmatrix** out);
/* Uploads rows [row_begin, row_end) only: the column shard a rank holds when
 * the output dimension N is split across GPUs. */
MRI_API int mri_qmatrix_upload_rows(mri_ctx* ctx, const int8_t* data, const float* scales,
                            size_t n_out, size_t k_in, size_t row_begin, size_t row_end,
                            mri_qmatrix** out);
MRI_API int mri_qmatrix_free(mri_qmatrix* w);
MRI_API int mri_qmatrix_dims(const mri_qmatrix* w, size_t* n_out, size_t* k_in);

/* Q8_0WeightMatrix::from_raw_bytes (q8_direct.rs:80-107): k_in % 32 == 0 and
 * len == n_out*(k_in/32)*34, else MRI_ERR_INVALID_SHAPE. */
MRI_API int mri_q8_0_upload(mri_ctx* ctx, const uint8_t* bytes, size_t len, size_t n_out,
                    size_t k_in, mri_q8_0_matrix** out);
MRI_API int mri_q8_0_free(mri_q8_0_matrix* w);
/* Q4_0 byte slice of a [n_out, k] matrix (q4_0.rs:8-21); the same k % 32 and
 * byte-length checks as matmul_q4_0_dequant (q4_0.rs:121-140). */
MRI_API int mri_q4_0_upload(mri_ctx* ctx, const uint8_t* bytes, size_t len, size_t n_out,
                    size_t k, mri_q4_0_matrix** out);
MRI_API int mri_q4_0_free(mri_q4_0_matrix* w);

/* ── GGUF tensor data to device weights ───────────────────────────────────── */
/* ggml storage types TensorExtractor::extract accepts (gguf/dtype.rs:30-43,
 * extract.rs:728-732). */
#define MRI_GGML_F32 0
#define MRI_GGML_F16 1
#define MRI_GGML_Q4_0 2
#define MRI_GGML_Q8_0 8
/* quantize_tensor(&extractor.extract(name)) (forward_int8.rs:52-62 with
 * extract.rs:719-737): `bytes` is the tensor's raw GGUF data in host memory
 * (e.g. a slice of the mapped file), [n_out, k_in] its row-major shape (GGUF
 * dims reversed, tensor_info.rs:145-147).  The bytes are copied to the device
 * and dequantized and requantized per output row there; the result is
 * bit-identical to dequantize-then-quantize_per_channel on the host.
 * Unsupported type -> MRI_ERR_INVALID_ARGUMENT (GgufError::TypeMismatch);
 * n_out*k_in not a multiple of 32 for Q8_0/Q4_0, or len not the type's byte
 * count -> MRI_ERR_SHAPE_MISMATCH (GgufError::ShapeMismatch).  Synchronous. */
MRI_API int mri_qmatrix_from_gguf(mri_ctx* ctx, int ggml_type, const uint8_t* bytes, size_t len,
                                  size_t n_out, size_t k_in, mri_qmatrix** out);
/* Copies a matrix's rows and scales back to host memory (the data / scales
 * fields of QuantizedMatrix, per_channel.rs:29-40).  Synchronous. */
MRI_API int mri_qmatrix_download(const mri_qmatrix* w, int8_t* data, float* scales);
/* TensorExtractor::extract (extract.rs:719-737) into device memory: numel f32
 * values at out_dev.  Same checks as mri_qmatrix_from_gguf.  Synchronous. */
MRI_API int mri_gguf_dequant(mri_ctx* ctx, int ggml_type, const uint8_t* bytes, size_t len,
                             size_t numel, float* out_dev);

/* ── activation quantizer (quantize_symmetric, symmetric.rs:42-57) ────────── */
/* x_dev [m,k] f32 -> q_dev [m,k] i8 and scale_dev (1 value for PER_TENSOR,
 * m values for PER_ROW). */
MRI_API int mri_quantize_symmetric(mri_ctx* ctx, const float* x_dev, size_t m, size_t k,
                           int granularity, int8_t* q_dev, float* scale_dev);

/* ── INT8 x INT8 -> INT32 -> f32 (int8.rs / int8_avx2.rs / parallel.rs) ──── */
/* matmul_int8(act_q, act_scale, weights, m) (int8.rs:61-98; same contract as
 * matmul_int8_avx2 int8_avx2.rs:174, matmul_int8_neon int8_neon.rs:158 and
 * matmul_int8_parallel parallel.rs:308).  act_len != m*k_in -> INVALID_SHAPE.
 * out_dev [m,n] f32; acc_dev (nullable) receives the i32 accumulators. */
MRI_API int mri_matmul_int8(mri_ctx* ctx, const int8_t* act_q_dev, size_t act_len, float act_scale,
                    const mri_qmatrix* w, size_t m, float* out_dev, int32_t* acc_dev);
/* Same, with the activation scale(s) already on the device: one value, or m
 * values when scale_per_row != 0. */
MRI_API int mri_matmul_int8_dscale(mri_ctx* ctx, const int8_t* act_q_dev, size_t act_len,
                           const float* act_scale_dev, int scale_per_row,
                           const mri_qmatrix* w, size_t m, float* out_dev, int32_t* acc_dev);
/* matmul_int8_from_f32(input, weights) (int8.rs:113-143): k != k_in ->
 * SHAPE_MISMATCH; per-tensor quantization of the whole [m,k] input, fused. */
MRI_API int mri_matmul_int8_from_f32(mri_ctx* ctx, const float* x_dev, size_t m, size_t k,
                             const mri_qmatrix* w, float* out_dev);
/* Explicit-granularity variant (MRI_PER_ROW quantizes each input row on its
 * own, the form BASELINE's prefill config describes). */
MRI_API int mri_matmul_int8_from_f32_g(mri_ctx* ctx, const float* x_dev, size_t m, size_t k,
                               int granularity, const mri_qmatrix* w, float* out_dev);

/* ── block-quantized products ─────────────────────────────────────────────── */
/* matmul_q8_0_direct(input, weights) (q8_direct.rs:229-289): per-row
 * activation quantization, per-block i32 dot, f32 accumulation over blocks
 * in block order (bit-exact with the reference). */
MRI_API int mri_matmul_q8_0_direct(mri_ctx* ctx, const float* x_dev, size_t m, size_t k,
                           const mri_q8_0_matrix* w, float* out_dev);
/* matmul_q4_0_dequant(input, weight_q4, n_out, k) (q4_0.rs:94-181): f32 x
 * dequantized nibbles, f32 accumulation (tolerance, not bit-exact: the sum
 * is reassociated across the warp). */
MRI_API int mri_matmul_q4_0_dequant(mri_ctx* ctx, const float* x_dev, size_t m, size_t k,
                            const mri_q4_0_matrix* w, float* out_dev);

/* ── host-buffer drop-ins (synchronous) ───────────────────────────────────── */
MRI_API int mri_host_quantize_symmetric(mri_ctx* ctx, const float* x, size_t m, size_t k,
                                int granularity, int8_t* q, float* scale);
MRI_API int mri_host_matmul_int8(mri_ctx* ctx, const int8_t* act_q, size_t act_len, float act_scale,
                         const mri_qmatrix* w, size_t m, float* out, int32_t* acc);
MRI_API int mri_host_matmul_int8_from_f32(mri_ctx* ctx, const float* x, size_t m, size_t k,
                                  const mri_qmatrix* w, float* out);
MRI_API int mri_host_matmul_q8_0_direct(mri_ctx* ctx, const float* x, size_t m, size_t k,
                                const mri_q8_0_matrix* w, float* out);
MRI_API int mri_host_matmul_q4_0_dequant(mri_ctx* ctx, const float* x, size_t m, size_t k,
                                 const mri_q4_0_matrix* w, float* out);

/* ── LlamaModelInt8 (model/llama/forward_int8.rs:416-547) ────────────────── */
/* The device-resident model around the projections: flat f32 KV cache
 * [layer][max_seq][kv_dim], per-tensor INT8 projections (Q/K/V and gate/up
 * stored concatenated; bit-identical per element to separate calls), f32
 * RMSNorm / RoPE / causal GQA attention / SwiGLU / residual glue. */
typedef struct mri_llama mri_llama;
typedef struct mri_llama_config {
  uint32_t n_layers, dim, n_heads, n_kv_heads /* 0 = n_heads */, ffn_dim, vocab, max_seq;
  float rope_base, rms_eps;
} mri_llama_config;
MRI_API int mri_llama_create(mri_ctx* ctx, const mri_llama_config* cfg, mri_llama** out);
MRI_API int mri_llama_free(mri_llama* m);
MRI_API const char* mri_llama_last_error(void);
/* Weights from host memory (LlamaModelInt8::new, forward_int8.rs:427-440). */
MRI_API int mri_llama_set_rope(mri_llama* m, const float* cos_t, const float* sin_t); /* [max_seq, hd/2] */
MRI_API int mri_llama_set_embedding(mri_llama* m, const float* token_embd);        /* [vocab, dim] */
MRI_API int mri_llama_set_norms(mri_llama* m, const float* attn_norm /*[L,dim]*/,
                                const float* ffn_norm /*[L,dim]*/, const float* output_norm);
MRI_API int mri_llama_set_layer(mri_llama* m, uint32_t layer, const int8_t* wq, const float* sq,
                                const int8_t* wk, const float* sk, const int8_t* wv, const float* sv,
                                const int8_t* wo, const float* so, const int8_t* wgate,
                                const float* sgate, const int8_t* wup, const float* sup,
                                const int8_t* wdown, const float* sdown);
MRI_API int mri_llama_set_output(mri_llama* m, const int8_t* w, const float* s); /* [vocab, dim] */
/* Weights from a GGUF file (LlamaModelInt8::from_loader, forward_int8.rs:461-507):
 * one tensor's raw GGUF data in host memory, stored as MRI_GGML_F32 / F16 /
 * Q8_0 / Q4_0, row-major shape [rows, cols] (a 1-D tensor of d values is
 * [1, d]).  Projections and the output matrix are dequantized and requantized
 * per output row on the device (quantize_tensor of extract, bit-identical to
 * the host path); the embedding and the norm vectors are dequantized to f32
 * on the device.  Roles follow weight_name / global_weight_name
 * (model/llama/weights.rs:62-104); `layer` is ignored for the three global
 * tensors.  A shape other than the configuration's -> MRI_ERR_SHAPE_MISMATCH;
 * type and byte-length errors as mri_qmatrix_from_gguf.  Synchronous. */
enum {
  MRI_TENSOR_TOKEN_EMBD = 0, /* token_embd.weight  [vocab, dim] */
  MRI_TENSOR_OUTPUT_NORM = 1, /* output_norm.weight [dim] */
  MRI_TENSOR_OUTPUT = 2,     /* output.weight      [vocab, dim] */
  MRI_TENSOR_ATTN_Q = 3,     /* blk.L.attn_q.weight      [n_heads*hd, dim] */
  MRI_TENSOR_ATTN_K = 4,     /* blk.L.attn_k.weight      [n_kv*hd, dim] */
  MRI_TENSOR_ATTN_V = 5,     /* blk.L.attn_v.weight      [n_kv*hd, dim] */
  MRI_TENSOR_ATTN_OUTPUT = 6, /* blk.L.attn_output.weight [dim, n_heads*hd] */
  MRI_TENSOR_ATTN_NORM = 7,  /* blk.L.attn_norm.weight   [dim] */
  MRI_TENSOR_FFN_GATE = 8,   /* blk.L.ffn_gate.weight    [ffn, dim] */
  MRI_TENSOR_FFN_UP = 9,     /* blk.L.ffn_up.weight      [ffn, dim] */
  MRI_TENSOR_FFN_DOWN = 10,  /* blk.L.ffn_down.weight    [dim, ffn] */
  MRI_TENSOR_FFN_NORM = 11   /* blk.L.ffn_norm.weight    [dim] */
};
MRI_API int mri_llama_load_tensor(mri_llama* m, int role, uint32_t layer, int ggml_type,
                                  const uint8_t* bytes, size_t len, size_t rows, size_t cols);
/* Synthetic weights generated on the device (benchmarking only). */
MRI_API int mri_llama_init_random(mri_llama* m, uint64_t seed);
/* LlamaModelInt8::forward (forward_int8.rs:516-529): logits [n, vocab]; also
 * fills the KV cache for positions [0, n).
 * Prefill attention runs on the tensor cores with q, k and v split into f16
 * high and low parts.  A call that meets a q, k or v value beyond the f16
 * range (|v| > 65504) or a NaN is run again with the f32 CUDA-core attention
 * (mri_llama_attention_fallbacks counts such calls); this holds for
 * mri_llama_forward_at and mri_llama_generate_greedy too. */
MRI_API int mri_llama_forward(mri_llama* m, const uint32_t* tokens, size_t n, float* logits);
/* The block loop of TransformerBlockInt8::forward_cached_parallel
 * (forward_int8.rs:232-249, with forward_cached :206-215) at start_pos for
 * every layer, then the output norm and head: the n tokens take positions
 * [start_pos, start_pos + n), their K/V rows are written to the cache there,
 * and each attends to cache rows [0, its position] — rows [0, start_pos)
 * must hold an earlier prefill or decode of the same sequence.  Logits
 * [n, vocab].  start_pos + n > max_seq -> MRI_ERR_INVALID_SHAPE.  (The
 * reference's MIN_PARALLEL_SEQ switch, :243-246, only chooses its thread
 * schedule; both of its paths give the same numbers, as does this one.) */
MRI_API int mri_llama_forward_at(mri_llama* m, const uint32_t* tokens, size_t n, size_t start_pos,
                                 float* logits);
/* TransformerBlockInt8::forward_cached_parallel(x, start_pos, cache, layer)
 * (forward_int8.rs:232-249; equal to forward_cached :206-215): one block of
 * layer `layer` on the host input x [n, dim] at positions [start_pos,
 * start_pos + n), with the model's KV cache standing for `cache[layer]`
 * (rows written there, rows [0, start_pos) read).  out [n, dim] (may alias
 * x).  Synchronous.  layer >= n_layers, n == 0 or start_pos + n > max_seq ->
 * MRI_ERR_INVALID_SHAPE. */
MRI_API int mri_llama_block_forward(mri_llama* m, uint32_t layer, const float* x, size_t n,
                                    size_t start_pos, float* out);
/* LlamaModelInt8::forward_decode (forward_int8.rs:538-546): logits [vocab]. */
MRI_API int mri_llama_forward_decode(mri_llama* m, uint32_t token, size_t pos, float* logits);
/* Prefill the prompt into the cache (an addition: the reference has no
 * cached prefill at model level), then n_decode greedy steps replayed from a
 * captured CUDA graph.  out_tokens receives n_decode + 1 tokens (the first
 * from the prompt's last logits).  Device-timed prefill / decode in ms. */
MRI_API int mri_llama_generate_greedy(mri_llama* m, const uint32_t* prompt, size_t n_prompt,
                                      size_t n_decode, uint32_t* out_tokens, float* prefill_ms,
                                      float* decode_ms);
MRI_API int mri_llama_launches_per_decode_step(const mri_llama* m, size_t* count);
/* No counterpart in the reference.  A model starts with the kernel-variant
 * options of the context it was created on; this sets one for the model
 * alone (mri_ctx_set_option semantics; a captured decode graph keeps the
 * variant it was captured with). */
MRI_API int mri_llama_set_option(mri_llama* m, int option, int value);
/* No counterpart in the reference.  Calls run again with the f32 prefill
 * attention because a q, k or v value left the f16 range. */
MRI_API int mri_llama_attention_fallbacks(const mri_llama* m, size_t* count);

/* ── allocation-free entry point ───────────────────────────────────────────── */
/* No counterpart in the reference.  For callers that cannot allocate device
 * memory at call time (a host runtime that owns the device memory pool and
 * forbids cudaMalloc/cudaFree, or code that must not touch an allocator while
 * a framework manages the stream): matmul_int8_from_f32 with per-tensor
 * quantization, whose scratch (quantized activations, absmax, scale, status
 * word) lives in a fixed file-scope device array instead of a context buffer.
 * 1..8 rows run on the streaming GEMV, more on the tensor-core GEMM; the
 * result equals mri_matmul_int8_from_f32 bit for bit.
 *   - Takes raw device pointers and a cudaStream_t (NULL = legacy stream);
 *     needs no context.  w_dev: [n,k] int8 row-major (16-byte aligned),
 *     w_scales_dev: [n] f32, x_dev: [m,k] f32, out_dev: [m,n] f32.
 *   - m*k must not exceed MRI_NOALLOC_MAX_ACT_BYTES, else
 *     MRI_ERR_INVALID_ARGUMENT before any work; k must be a positive multiple
 *     of 16.
 *   - The first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress) and device properties and clears the status
 *     word; make that first call before any stream capture.
 *   - All calls share the one array: calls that overlap on the GPU (other
 *     streams, other threads) race.  Serialize them on one stream.
 *   - Every GPU that loads this library keeps the array allocated until the
 *     process exits.
 *   - The call is asynchronous, and a bounded device-side wait that gives up
 *     cannot change its return value: it records MRI_ERR_TIMEOUT in the
 *     array's status word (the output is then incomplete).  The word stays
 *     set until mri_noalloc_check_status(stream) synchronizes `stream`, reads
 *     it into host memory, clears it and returns it (MRI_OK or
 *     MRI_ERR_TIMEOUT); call it before using outputs that must be complete.
 *   - Errors: mri_noalloc_last_error(). */
#define MRI_NOALLOC_MAX_ACT_BYTES (4u << 20)
MRI_API int mri_matmul_int8_from_f32_noalloc(const float* x_dev, size_t m, size_t k,
                                             const int8_t* w_dev, const float* w_scales_dev,
                                             size_t n, float* out_dev, void* cuda_stream);
MRI_API int mri_noalloc_check_status(void* cuda_stream);
MRI_API const char* mri_noalloc_last_error(void);

/* ── N-sharded products over NCCL ───────────────────────────────────────────── */
/* No counterpart in the reference (it runs on one host).  For weight matrices
 * split across the GPUs of one node, one process (or thread) per GPU: rank r
 * of P holds rows [r*N/P, (r+1)*N/P) of W (mri_shard_rows, then
 * mri_qmatrix_upload_rows), and mri_sharded_matmul_int8_from_f32 returns the
 * full [m, N] product on every rank, bit-identical to the unsharded
 * mri_matmul_int8_from_f32 (same kernels per element, per-tensor activation
 * scale over the whole input on every rank, NCCL all-gather of f32 slices).
 *   - NCCL is loaded at run time (libnccl.so.2); mri_comm_available() says
 *     whether it could be.  Rank 0 calls mri_comm_unique_id and the host
 *     application sends the MRI_COMM_ID_BYTES bytes to the other ranks.
 *   - mri_comm_create binds the communicator to the context's device and
 *     stream.  Host-side waits (creation, enqueue, mri_comm_wait) give up
 *     after timeout_ms (<= 0: 60 s), abort the communicator and return
 *     MRI_ERR_TIMEOUT; an aborted communicator refuses further calls.
 *   - mri_sharded_matmul_int8_from_f32 is asynchronous on the context's
 *     stream; x_dev [m,k] f32, out_dev [m,n_total] f32.  For m > 1 the rows
 *     are processed in chunks whose all-gathers overlap the next chunk's
 *     product; the staging buffer grows on demand (a growth synchronizes).
 *     N % P != 0 -> MRI_ERR_INVALID_SHAPE, wrong shard height or k ->
 *     MRI_ERR_SHAPE_MISMATCH, NCCL failures -> MRI_ERR_COMM.
 *   - mri_comm_wait synchronizes the context's stream and the communicator's
 *     side stream, watching NCCL's asynchronous error state. */
typedef struct mri_comm mri_comm;
#define MRI_COMM_ID_BYTES 128
MRI_API int mri_comm_available(void);
MRI_API int mri_comm_unique_id(uint8_t* id /* [MRI_COMM_ID_BYTES] */);
MRI_API int mri_comm_create(mri_ctx* ctx, const uint8_t* id, int nranks, int rank, int timeout_ms,
                            mri_comm** out);
MRI_API int mri_comm_destroy(mri_comm* comm);
MRI_API int mri_comm_rank(const mri_comm* comm, int* rank, int* nranks);
MRI_API int mri_comm_wait(mri_comm* comm);
MRI_API int mri_shard_rows(size_t n, int nranks, int rank, size_t* row_begin, size_t* row_end);
MRI_API int mri_sharded_matmul_int8_from_f32(mri_comm* comm, const float* x_dev, size_t m, size_t k,
                                             const mri_qmatrix* w_shard, size_t n_total,
                                             float* out_dev);

/* ── diagnostics ──────────────────────────────────────────────────────────── */
/* No counterpart in the reference (its dot kernel is routed by target
 * architecture at build time, src/ops/matmul/parallel.rs:258-275).
 * Kernel path chosen for an INT8 product of this shape:
 * 0 = streaming GEMV (TMA bulk), 1 = generic GEMV, 2 = tensor-core GEMM. */
MRI_API int mri_int8_path(mri_ctx* ctx, size_t m, size_t n, size_t k);
/* Launch shape of the streaming INT8 GEMV for (m <= 8, n, k): plan[0..7] =
 * grid, CTAs per SM used, CTAs per SM that fit (registers and shared
 * memory), pipeline stages, K-chunks per row group, dynamic shared bytes,
 * register-prologue width of a per-tensor f32 input (4 or 12 float4 per
 * consumer thread, 0 = none), and 1 when such an input is quantized by the
 * quantizer kernels first (then the GEMV streams int8 activations). */
MRI_API int mri_int8_gemv_plan(mri_ctx* ctx, size_t m, size_t n, size_t k, int* plan /* [8] */);
/* Launch shape of the tensor-core INT8 GEMM for (m, n, k) with a plain
 * output (no residual, no INT32 copy): plan[0..6] = tile width BN, ring
 * stages, TMEM accumulator buffers per CTA (2: persistent grid, each CTA (or
 * CTA pair) walks tiles t, t + grid, ...; 1: one tile per CTA, two CTAs per
 * SM), grid (CTAs), tiles, the most tiles one CTA (pair) takes, and 2 when
 * CTA pairs run 256-row tiles on tcgen05.mma.cta_group::2 (else 1).  Follows
 * the context's options.  No tensor-core GEMM -> MRI_ERR_INVALID_SHAPE. */
MRI_API int mri_int8_gemm_plan(mri_ctx* ctx, size_t m, size_t n, size_t k, int* plan /* [7] */);

#ifdef __cplusplus
}
#endif
#endif /* MRI_GPU_H */
