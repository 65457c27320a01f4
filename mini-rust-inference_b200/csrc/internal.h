// internal.h — launch interfaces between the ABI layer (abi.cu) and the
// kernel translation units.  Not part of the public C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

struct mri_ctx;
struct mri_qmatrix;

namespace mri {

// Where the activations of a product come from.
enum ActMode : int {
  ACT_F32_PER_TENSOR = 0,  // x f32 [M,K]: quantize with one scale over all M*K values
  ACT_F32_PER_ROW = 1,     // x f32 [M,K]: quantize each row with its own scale
  ACT_I8_HOST_SCALE = 2,   // xq i8 [M,K] + one scale passed by value
  ACT_I8_DEV_SCALE = 3,    // xq i8 [M,K] + one scale in device memory
  ACT_I8_DEV_ROW_SCALE = 4 // xq i8 [M,K] + M scales in device memory
};

struct ActArgs {
  const float* x = nullptr;
  const int8_t* xq = nullptr;
  const float* scale_dev = nullptr;
  float scale_host = 1.0f;
  int mode = ACT_F32_PER_TENSOR;
  // Optional producer ops fused in front of the f32 quantization (modes 0/1):
  //   norm_w: RMSNorm of each row (ops/norm/rmsnorm.rs:51-117) with weight
  //           norm_w [K] and epsilon eps, before quantization;
  //   swiglu: the input rows are 2K wide with gate and up interleaved
  //           (element k: gate at 2k, up at 2k+1) and the quantized value is
  //           silu(gate) * up (ops/activation/swiglu.rs:39-61).
  const float* norm_w = nullptr;
  float eps = 0.0f;
  int swiglu = 0;
  // Streaming GEMV: weight stages the producer issues before the activation
  // loads are in flight (-1: one).  A projection that follows a kernel which
  // leaves HBM mostly idle (decode attention) prefetches its whole ring.
  int pre_stages = -1;
};

// Optional epilogues of the streaming INT8 GEMV that combine adjacent output
// rows (2i, 2i+1) of the same activation row.  Both need N even.
enum EpiMode : int {
  EPI_NONE = 0,
  // out[m, i] = silu(y[m, 2i]) * y[m, 2i+1]  (gate/up rows interleaved; out
  // is [M, N/2]; ops/activation/swiglu.rs:39-61).
  EPI_SWIGLU = 1,
  // Fused QKV rows [q (qd) | k (kvd) | v (kvd)]: q and k rotated in adjacent
  // pairs at position pos + m (ops/rope.rs:121-190; pos = *pos_dev when given,
  // else pos0), written to out; rotated k and plain v also written to the
  // cache rows kc/vc [pos + m] (attention/cached.rs:90-93).
  EPI_ROPE_KV = 2,
  // N-sharded product gathered over peer memory (no NCCL): each CTA writes its
  // output rows into the staging buffer of every rank ([2][M][n_total], half =
  // parity of the call count, columns of rank r at [r*N, (r+1)*N)) and counts
  // itself in on every rank's arrival counter; launch_gather_collect then
  // waits for all ranks and copies the staged result to `g_out`.
  EPI_GATHER = 3,
};

struct EpiArgs {
  int mode = EPI_NONE;
  const int* pos_dev = nullptr;
  int pos0 = 0;
  const float* cos_t = nullptr;  // [max_seq, hd/2]
  const float* sin_t = nullptr;
  int hd = 0, qd = 0, kvd = 0;
  float* kc = nullptr;  // [max_seq, kvd]
  float* vc = nullptr;
  // EPI_GATHER
  static constexpr int kMaxRanks = 8;
  float* g_stage[kMaxRanks] = {};              // per rank (peer pointers)
  unsigned long long* g_ctr[kMaxRanks] = {};   // per rank arrival counters
  unsigned long long* g_seq = nullptr;         // local call state, 4 words (gemv.cu)
  size_t g_half = 0;                           // floats per staging half
  size_t g_ntotal = 0;
  int g_ranks = 1, g_rank = 0;
  float* g_out = nullptr;
};

// Kernel counts for launch accounting.
struct LaunchStats {
  unsigned long long launches = 0;
};

// Kernel-variant options of a context (mri_ctx_set_option).  The defaults are
// the measured best choices; the others exist so that every variant the
// launchers can take is reachable, and tested, without a rebuild.  They are
// set explicitly through the C ABI, never read from the environment.
struct Options {
  int pdl = 1;         // MRI_OPT_PDL: programmatic dependent launch between kernels
  int gemm_bn = 0;     // MRI_OPT_GEMM_BN: 0 = tile width per shape, else 128..256 step 32
  int gemm_2cta = 1;   // MRI_OPT_GEMM_2CTA: one tile per CTA, two CTAs per SM, between one and two rounds of tiles
  int q8_mma = 1;      // MRI_OPT_Q8_MMA: Q8_0 at m = 2..8 on the integer warp MMA
  int q4_mma = 1;      // MRI_OPT_Q4_MMA: Q4_0 at m = 2..8 on the bf16 warp MMA
  int tc_attn = 1;     // MRI_OPT_TC_ATTN: tensor-core prefill attention (head dim 64 / 128)
  int fa_split = 3;    // MRI_OPT_FA_SPLIT: key tiles from which a prefill key walk is split (0 = never)
  int shard_peer = 2;  // MRI_OPT_SHARD_PEER: 0 NCCL, 1 peer memory, 2 peer memory for m > 8 only
  int gemm_pair = 1;   // MRI_OPT_GEMM_PAIR: 1 CTA pairs from 4 rounds of pair tiles, 2 always, 0 never
  int q4_limb = 1;     // MRI_OPT_Q4_LIMB: Q4_0 at m = 1 on integer block dots
  // Internal (not an ABI option): SMs the tensor-core GEMM leaves free for
  // other work running beside it.
  int sm_reserve = 0;
};

// Per-device properties the launchers need, and the context's options.
struct DeviceInfo {
  int device = 0;
  int sm_count = 0;
  int max_smem_optin = 0;
  int cc_major = 0, cc_minor = 0;
  size_t l2_bytes = 0;
  Options opt;
};

// ── quantizer (quant.cu) ─────────────────────────────────────────────────────
// amax_scratch: 2 * max(M, kQuantPartials) floats of device scratch (per-block
// partial maxima for PER_TENSOR, per-row maxima for PER_ROW, per-row 1/rms
// when norm_w is given).  sync (nullable): two zero-initialised words of
// device memory owned by the caller's stream, the grid barrier of the
// one-launch per-tensor quantizer; without them the two-kernel path runs.
// status: where a barrier wait that gives up records MRI_ERR_TIMEOUT.
constexpr size_t kQuantPartials = 1024;
cudaError_t launch_quantize(const DeviceInfo& dev, cudaStream_t st, const float* x, size_t m,
                            size_t k, int per_row, int8_t* q, float* scale, float* amax_scratch,
                            LaunchStats* ls, const float* norm_w = nullptr, float eps = 0.0f,
                            int swiglu = 0, unsigned* sync = nullptr, int* status = nullptr);

// out[i] = residual[i] + out[i] (the reference's x + projected).
// n floats (n % 4 == 0, both 16-byte aligned) from device memory into a
// pinned host buffer's device mapping, after the previous kernel in the stream.
cudaError_t launch_copy_out(const DeviceInfo& dev, cudaStream_t st, const float* src, float* dst,
                            size_t n, LaunchStats* ls);
cudaError_t launch_add_residual(const DeviceInfo& dev, cudaStream_t st, float* out,
                                const float* residual, size_t n, LaunchStats* ls);

// ── streaming GEMV family (gemv.cu), M <= 8 rows of activations ─────────────
// INT8 per-channel.  Requires K % 16 == 0 and 16-byte aligned W.
bool gemv_i8_tma_supported(const DeviceInfo& dev, int M, size_t K);
// residual (nullable): out = residual + product, element-wise (may alias out).
// Register-prologue width (float4 per consumer thread: 4 or 12) the INT8
// streaming GEMV uses for this input, 0 when the input takes the general path.
int reg_vec(int M, size_t K, const ActArgs* act);
// Launch shape the INT8 streaming GEMV uses for (M, N, K).
struct GemvPlan {
  int grid = 0, ctas_per_sm = 0, resident = 0, stages = 0, k_chunks = 0, vec = 0;
  int epi = 0;
  size_t smem = 0;
};
// vec < 0: the register-path width of a plain per-tensor f32 input.
// epi_kind: 0 none, 1 pair epilogue (M = 1), 2 peer gather.
cudaError_t gemv_i8_tma_plan(const DeviceInfo& dev, int M, size_t N, size_t K, GemvPlan* plan,
                             int vec = -1, int epi_kind = 0);
// epi (nullable): a pair epilogue (EpiArgs); not combined with residual or acc_out.
cudaError_t launch_gemv_i8_tma(const DeviceInfo& dev, cudaStream_t st, int M, const int8_t* W,
                               const float* w_scales, size_t N, size_t K, const ActArgs& act,
                               float* out, int32_t* acc_out, int* status, LaunchStats* ls,
                               const float* residual = nullptr, const EpiArgs* epi = nullptr);
// Second kernel of an EPI_GATHER product: waits (bounded) for every rank's
// arrivals of the preceding gather GEMV and copies [M][n_total] to e.g_out.
cudaError_t launch_gather_collect(const DeviceInfo& dev, cudaStream_t st, const EpiArgs& e, int M,
                                  int* status, LaunchStats* ls);
// Any K, any alignment; activations must be pre-quantized (modes 2-4).
cudaError_t launch_gemv_i8_generic(const DeviceInfo& dev, cudaStream_t st, int M, const int8_t* W,
                                   const float* w_scales, size_t N, size_t K, const ActArgs& act,
                                   float* out, int32_t* acc_out, LaunchStats* ls);

// Q8_0 (34-byte blocks).  Per-row activation quantization is fused.
bool gemv_q8_0_tma_supported(const DeviceInfo& dev, int M, size_t K);
cudaError_t launch_gemv_q8_0_tma(const DeviceInfo& dev, cudaStream_t st, int M, const uint8_t* W,
                                 size_t N, size_t K, const float* x, float* out, int* status,
                                 LaunchStats* ls);
// M = 2..8: block dots on the warp MMA.  act is ACT_I8_DEV_ROW_SCALE: the
// rows quantized per row beforehand (xq [M, K] and M scales on the device).
// q8_0_mma_supported tells where the kernel applies.
bool q8_0_mma_supported(const DeviceInfo& dev, int M, size_t K);
cudaError_t launch_gemv_q8_0_mma(const DeviceInfo& dev, cudaStream_t st, int M, const uint8_t* W,
                                 size_t N, size_t K, const ActArgs& act, float* out, int* status,
                                 LaunchStats* ls);
// Generic: activations pre-quantized per row into xq/scales (device).
cudaError_t launch_gemv_q8_0_generic(const DeviceInfo& dev, cudaStream_t st, int M,
                                     const uint8_t* W, size_t N, size_t K, const int8_t* xq,
                                     const float* scales, float* out, LaunchStats* ls);

// Q4_0 (18-byte blocks), f32 activations.
// M = 2..8 on the bf16 warp MMA: launch_q4_0_split writes x [m, K] (16-byte
// aligned) as split bf16 pairs in fragment order (q4_0_split_bytes(m, K)
// bytes, 16-byte aligned; a chunk of rows starts at row * q4_0_split_bytes(1,
// K)), which launch_gemv_q4_0_mma then reads.
bool q4_0_mma_supported(const DeviceInfo& dev, int M, size_t K);
size_t q4_0_split_bytes(size_t m, size_t K);
cudaError_t launch_q4_0_split(const DeviceInfo& dev, cudaStream_t st, const float* x, size_t m,
                              size_t K, uint32_t* xs, LaunchStats* ls);
cudaError_t launch_gemv_q4_0_mma(const DeviceInfo& dev, cudaStream_t st, int M, const uint8_t* W,
                                 size_t N, size_t K, const uint32_t* xs, float* out, int* status,
                                 LaunchStats* ls);
bool gemv_q4_0_tma_supported(const DeviceInfo& dev, int M, size_t K);
// M = 1, K % 1024 == 0, x 16-byte aligned: integer block dots (f32 for a
// row with an inf or a NaN).
bool gemv_q4_0_limb_supported(const DeviceInfo& dev, size_t K, const float* x);
cudaError_t launch_gemv_q4_0_limb(const DeviceInfo& dev, cudaStream_t st, const uint8_t* W, size_t N,
                                  size_t K, const float* x, float* out, int* status, LaunchStats* ls);
cudaError_t launch_gemv_q4_0_tma(const DeviceInfo& dev, cudaStream_t st, int M, const uint8_t* W,
                                 size_t N, size_t K, const float* x, float* out, int* status,
                                 LaunchStats* ls);
cudaError_t launch_gemv_q4_0_generic(const DeviceInfo& dev, cudaStream_t st, int M,
                                     const uint8_t* W, size_t N, size_t K, const float* x,
                                     float* out, LaunchStats* ls);

// INT8 product of an f32 [m, k] input with per-tensor quantization and the
// optional fused producer ops of ActArgs (RMSNorm or SwiGLU; for SwiGLU the
// input rows are 2k wide) and residual epilogue.  `epi` (nullable) selects a
// pair epilogue; it is only available for one activation row on the
// streaming GEMV path (matmul_int8_epilogue_supported).  Status code as the
// C ABI.
int matmul_int8_fused(struct ::mri_ctx* ctx, const float* x, size_t m, size_t k,
                      const float* norm_w, float eps, int swiglu,
                      const struct ::mri_qmatrix* w, const float* residual, float* out,
                      const EpiArgs* epi = nullptr, int pre_stages = -1);
// Records the calling thread's last error (mri_last_error) and returns code.
int set_error(int code, const char* fmt, ...);
// Per-tensor quantization of x [m, k] into the context scratch (quantized
// values and one device scale), for callers that run several products on
// slices of the same quantized input.
int quantize_to_scratch(struct ::mri_ctx* ctx, const float* x, size_t m, size_t k, int8_t** q,
                        float** scale_dev);
// The INT8 dispatch (streaming GEMV / tensor-core GEMM) for any ActArgs mode.
int matmul_int8_act(struct ::mri_ctx* ctx, const ActArgs& act, const struct ::mri_qmatrix* w,
                    size_t m, float* out);
// The streaming GEMV serves an INT8 product of m activation rows with w.
bool stream_gemv_ok(const struct ::mri_ctx* ctx, size_t m, const struct ::mri_qmatrix* w);
// N-sharded product of x [m <= 8, k] with this rank's shard, gathered over
// peer memory (EPI_GATHER); e carries the gather fields.  Status as the C ABI.
int matmul_int8_gather(struct ::mri_ctx* ctx, const float* x, size_t m, size_t k,
                       const struct ::mri_qmatrix* w, const EpiArgs& e);
bool matmul_int8_epilogue_supported(const struct ::mri_ctx* ctx, size_t m,
                                    const struct ::mri_qmatrix* w);

// Grows the context scratch to at least `bytes` (synchronizes the stream
// when it reallocates).  Callers that capture CUDA graphs reserve their
// maximum first: a captured launch keeps the scratch address it saw.
int ctx_reserve_scratch(struct ::mri_ctx* ctx, size_t bytes);
// Scratch bytes an INT8 product with per-tensor quantization of an [m, k]
// input needs.
size_t int8_scratch_bytes(size_t m, size_t k);

// ── tensor-core INT8 GEMM (gemm_tc.cu) ──────────────────────────────────────
// Output of one GEMM call.  Plain: out [M][ldo] (ldo = N).  Gathered over
// peer memory (ranks > 1, an N-sharded product): the tile is written to `out`
// (this rank's columns of the full [M][n_total] output, i.e. out_full +
// rank * N, row stride ldo = n_total) and to every other rank's staging half
// (stage[p] + (seq & 1) * half + rank * N, same layout; seq = calls issued, in
// *g_seq (EpiArgs convention)); each CTA then counts itself in on every
// rank's arrival counter, and launch_gather_collect_cols copies the other
// ranks' columns out of this rank's staging.
struct GemmOut {
  float* out = nullptr;
  size_t ldo = 0;
  int ranks = 0, rank = 0;
  size_t half = 0, col0 = 0;
  float* stage[EpiArgs::kMaxRanks] = {};
  unsigned long long* ctr[EpiArgs::kMaxRanks] = {};
  unsigned long long* seq = nullptr;
};
bool gemm_i8_tc_supported(const DeviceInfo& dev, size_t M, size_t N, size_t K);
// Launch shape of the tensor-core GEMM for (M, N, K): tile width, ring
// stages, TMEM accumulator buffers per CTA (2: persistent grid, a CTA walks
// tiles t, t + grid, ...; 1: one tile per CTA, two CTAs per SM), grid,
// tiles, and the most tiles one CTA takes.
// pair = 2: two-CTA clusters issuing M = 256 MMAs (cta_group::2), tiles of
// 256 x bn (taken only for a plain output: no residual, no INT32 copy).
struct GemmPlan {
  int bn = 0, stages = 0, bufs = 0, grid = 0, tiles = 0, tiles_per_cta = 0, pair = 1;
};
cudaError_t gemm_i8_tc_plan(const DeviceInfo& dev, size_t M, size_t N, size_t K, GemmPlan* plan,
                            bool plain = true);
// xq [M,K] i8, W [N,K] i8 (both K-major), scale(s) in device memory.
cudaError_t launch_gemm_i8_tc(const DeviceInfo& dev, cudaStream_t st, const int8_t* xq,
                              const float* act_scale_dev, int scale_per_row, const int8_t* W,
                              const float* w_scales, size_t M, size_t N, size_t K, float* out,
                              int32_t* acc_out, int* status, LaunchStats* ls,
                              const float* residual = nullptr, const GemmOut* gather = nullptr);
// After a gathered GEMM: waits (bounded) for every rank's arrivals and copies
// the columns of the other ranks from this rank's staging into out_full
// [M][n_total] (this rank's own columns [rank * ns, (rank + 1) * ns) are
// already there).
cudaError_t launch_gather_collect_cols(const DeviceInfo& dev, cudaStream_t st, const GemmOut& g, size_t M,
                                       size_t ns, float* out_full, int* status, LaunchStats* ls);

// ── GGUF tensor data to device weights (load.cu) ────────────────────────────
// Destination of one converted tensor: either per-channel INT8 rows (row r ->
// q + r * q_stride, its scale -> scales[r * s_stride]) or, when f32 is set,
// the dequantized values (element i -> f32[i]).
struct GgufDst {
  int8_t* q = nullptr;
  size_t q_stride = 0;
  float* scales = nullptr;
  size_t s_stride = 1;
  float* f32 = nullptr;
};
// Bytes of `numel` elements stored as ggml type `type` (0 for other types).
size_t gguf_type_bytes(int type, size_t numel);
// TensorExtractor's type and length checks; status code as the C ABI and the
// reason in *err.
int gguf_check(int type, size_t len, size_t numel, std::string* err);
// Copies the host bytes of a [rows, cols] GGUF tensor to the device in steps
// of whole rows and converts them into `d` on stream `st`; returns after the
// last step has completed.
int gguf_to_device(cudaStream_t st, int type, const uint8_t* bytes, size_t len, size_t rows,
                   size_t cols, const GgufDst& d, std::string* err);

}  // namespace mri

// ── handle definitions shared by abi.cu and llama.cu ────────────────────────
struct mri_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  mri::DeviceInfo dev;
  int* d_status = nullptr;   // device view of the status word
  int* h_status = nullptr;   // host view (mapped pinned memory)
  unsigned* d_sync = nullptr;  // grid-barrier words of the one-launch quantizer (device memory)
  uint8_t* scratch = nullptr;
  size_t scratch_bytes = 0;
  mri::LaunchStats ls;
};

struct mri_qmatrix {
  int device;
  int8_t* data;
  float* scales;
  size_t n_out, k_in;
  bool owns = true;  // false when the storage belongs to a larger allocation
};

struct mri_q8_0_matrix {
  int device;
  uint8_t* data;
  size_t n_out, k_in;
};

struct mri_q4_0_matrix {
  int device;
  uint8_t* data;
  size_t n_out, k;
};
