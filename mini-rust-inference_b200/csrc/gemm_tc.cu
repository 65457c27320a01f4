// gemm_tc.cu — K3: INT8 x INT8 -> INT32 GEMM on the 5th-generation tensor
// cores (tcgen05.mma kind::i8, accumulators in TMEM) with the reference's
// rescale fused into the epilogue:  out[m,n] = ((f32)acc * s_a) * s_w[n]
// (ops/matmul/int8.rs:93, parallel.rs:340).
//
// C[M,N] = A[M,K] * B[N,K]^T with A = quantized activations and B = the
// QuantizedMatrix rows; both are K-major, which is the "TN" form tcgen05
// reads directly.  The INT32 sums are exact (no saturation), so the result
// is bit-identical to the reference's scalar loop.
//
// Persistent kernel, one CTA per SM, warp-specialised:
//   warp 0      : TMA producer.  2-D tiled loads (128-byte swizzle, no
//                 multicast) of a 128 x 128 A tile and a BN x 128 B tile per
//                 stage into a kStages-deep shared-memory ring.
//   warp 1      : allocates 2*BN TMEM columns (two accumulator buffers);
//                 one lane issues tcgen05.mma (M=128, N=BN, K=32 per
//                 instruction) and tcgen05.commit's stage releases and
//                 "accumulator ready" signals to mbarriers.
//   warps 2..5  : epilogue.  While a tile's MMAs run they stage its weight
//                 scales in shared memory; then tcgen05.ld of their 32-lane
//                 TMEM quarter (a thread per row), rescale, vectorised f32
//                 stores; the other accumulator buffer is being filled
//                 meanwhile.  (Scales read from global memory inside the
//                 chunk loop cost one L2 round trip per 4 columns there.)
// The producer issues the weight tiles of its first stages before
// griddepcontrol.wait (weights do not depend on the previous kernel) and the
// activation tiles after it.
// Every mbarrier wait is bounded; a timeout records MRI_ERR_TIMEOUT, raises
// a CTA-wide abort flag, drains in-flight copies / MMAs, frees TMEM, returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "internal.h"

namespace mri {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // K bytes per stage = one 128-byte swizzle row
constexpr int UMMA_K = 32;
constexpr int kEpiWarps = 4;
constexpr int kTcThreads = 32 * (2 + kEpiWarps);

// TMEM columns between the two accumulator buffers: a power of two, so both
// buffers start on an aligned column whatever the tile width.
template <int BN>
constexpr int acc_stride() { return BN <= 128 ? 128 : 256; }

// Output staging of the store epilogue: a 32 x 32 f32 block per epilogue warp.
constexpr size_t kStgBytes = kEpiWarps * 32 * 32 * 4;

template <int BN, int kStages, int kBufs = 2>
struct TcLayout {
  static constexpr size_t a_bytes = BM * BK;
  static constexpr size_t b_bytes = BN * BK;
  static constexpr size_t stage_bytes = a_bytes + b_bytes;
  // Weight scales of the tile, one buffer per accumulator buffer.
  static constexpr size_t epi = kStages * stage_bytes;
  static constexpr size_t epi_bytes = 2 * 256 * 4;
  // With one tile per CTA the stage ring is idle once the tile's MMAs are
  // done, and the epilogue stages its output there; otherwise it has its own.
  static constexpr size_t stg = kBufs == 1 ? 0 : epi + epi_bytes;
  static constexpr size_t bars = epi + epi_bytes + (kBufs == 1 ? 0 : kStgBytes);
  // full[S], empty[S], tfull[2], tempty[2], sready[2], mma_done, abort flag + tmem slot
  static constexpr size_t bars_bytes = (2 * kStages + 7) * 8 + 16;
  static constexpr size_t total = bars + bars_bytes + 1024;  // + alignment slack
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, int* status,
                                              volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (int i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0 && *abort_flag) return false;
    if (clock64() - t0 > kWaitBudgetClocks) {
      if (status) *reinterpret_cast<volatile int*>(status) = MRI_ERR_TIMEOUT;
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// K-major operand, 128-byte swizzle: rows of 128 bytes, 8-row atoms of 1024
// bytes (SBO), LBO unused (1), descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* p) {
  const uint32_t a = smem_addr(p);
  return (uint64_t((a >> 4) & 0x3FFF)) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::i8 instruction descriptor: D s32, A/B signed 8-bit, both K-major.
template <int BN>
__device__ __forceinline__ uint32_t idesc_i8() {
  return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// kBufs TMEM accumulator buffers: 2 for the persistent grid (tile t + 1's MMAs
// run while tile t is drained), 1 when every CTA takes exactly one tile and two
// CTAs share an SM (each holds half of the SM's 512 TMEM columns).
template <int BN, int kStages, int kBufs>
__global__ void __launch_bounds__(kTcThreads, kBufs == 1 ? 2 : 1)
    gemm_i8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const float* __restrict__ act_scale, int scale_per_row,
                      const float* __restrict__ w_scales, const __grid_constant__ GemmOut go,
                      int32_t* __restrict__ acc_out, int M, int N, int K, int* status,
                      const float* residual) {
  using L = TcLayout<BN, kStages, kBufs>;
  float* const out = go.out;
  const size_t ldo = go.ldo;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bars);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* sready = tempty + 2;
  uint64_t* mma_done = sready + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(mma_done + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1) + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
      mbar_init(&sready[b], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kBufs * acc_stride<BN>())
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: let the next kernel start early.  Nothing
  // a previous kernel may still be writing (activations, scales, residual) is
  // read before griddepcontrol.wait: the producer waits after issuing the
  // weight tiles of its first stages, the epilogue warps before their first
  // global read.  The MMA warp reads only shared memory and TMEM.  No-ops
  // without the launch attribute.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
      // Stage it holds k-block it % kblocks of this CTA's tile number it / kblocks.
      const int my_tiles = blockIdx.x < num_tiles ? (num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
      const int iters = my_tiles * kblocks;
      const int pre = std::min(kStages, iters);
      for (int it = 0; it < pre; ++it) {
        const int tile = blockIdx.x + (it / kblocks) * gridDim.x, kb = it % kblocks;
        uint8_t* sa = smem + it * L::stage_bytes;
        mbar_arrive_expect_tx(&full[it], static_cast<uint32_t>(L::stage_bytes));
        tma_load_2d(sa + L::a_bytes, &tmB, kb * BK, (tile / m_tiles) * BN, &full[it]);
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int it = 0; it < pre; ++it) {
        const int tile = blockIdx.x + (it / kblocks) * gridDim.x, kb = it % kblocks;
        tma_load_2d(smem + it * L::stage_bytes, &tmA, kb * BK, (tile % m_tiles) * BM, &full[it]);
      }
      int it = pre;
      for (; it < iters; ++it) {
        const int s = it % kStages;
        if (!wait_or_abort(&empty[s], ((it / kStages) - 1) & 1, status, abort_flag)) break;
        const int tile = blockIdx.x + (it / kblocks) * gridDim.x, kb = it % kblocks;
        uint8_t* sa = smem + s * L::stage_bytes;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(L::stage_bytes));
        tma_load_2d(sa, &tmA, kb * BK, (tile % m_tiles) * BM, &full[s]);
        tma_load_2d(sa + L::a_bytes, &tmB, kb * BK, (tile / m_tiles) * BN, &full[s]);
      }
      // Drain: every copy issued by this thread has landed before it exits.
      for (int j = std::max(0, it - kStages); j < it; ++j)
        mbar_wait(&full[j % kStages], (j / kStages) & 1, status);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_i8<BN>();
      int it = 0, t = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++t) {
        const int b = t & 1;
        if (t >= 2 && !wait_or_abort(&tempty[b], ((t >> 1) - 1) & 1, status, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * acc_stride<BN>();
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!wait_or_abort(&full[s], (it / kStages) & 1, status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* sa = smem + s * L::stage_bytes;
          const uint64_t adesc = smem_desc_sw128(sa);
          const uint64_t bdesc = smem_desc_sw128(sa + L::a_bytes);
#pragma unroll
          for (int j = 0; j < BK / UMMA_K; ++j)
            umma_i8(d_tmem, adesc + 2 * j, bdesc + 2 * j, idesc, (kb | j) != 0);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[b]);
      }
      // All MMAs issued by this thread are complete before TMEM is freed.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, status);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int et = threadIdx.x - 64;  // 0..127 among the epilogue warps
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const float s_all = scale_per_row ? 0.0f : ld_act(act_scale);
    const bool vec = (N % 4) == 0 && (ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(acc_out) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(residual) & 15) == 0 &&
                     (go.ranks <= 1 || (go.col0 % 4) == 0);
    // Gathered product: this call's staging half on the other ranks.
    const unsigned long long gseq = go.ranks > 1 ? ld_act(go.seq + 2) : 0ull;
    const size_t ghalf = (gseq & 1) * go.half;
    int t = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const int b = t & 1;
      const int m_blk = tile % m_tiles, n_blk = tile / m_tiles;
      const int row = m_blk * BM + q * 32 + lane;
      // Stage this tile's weight scales (the MMAs are still running).  Buffer
      // b was last read for tile t-2, which every warp finished before it
      // arrived on sready for tile t-1.
      float* s_sw = reinterpret_cast<float*>(smem + L::epi) + b * 256;
      for (int i = et; i < BN; i += 32 * kEpiWarps) {
        const int col = n_blk * BN + i;
        s_sw[i] = col < N ? __ldg(w_scales + col) : 0.0f;
      }
      const float s_a = scale_per_row ? (row < M ? ld_act(act_scale + row) : 0.0f) : s_all;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sready[b]);
      bool ok = wait_or_abort(&sready[b], (t >> 1) & 1, status, abort_flag);
      // Warp-uniform outcome: tcgen05.ld below is a .sync.aligned warp op.
      ok = ok && wait_or_abort(&tfull[b], (t >> 1) & 1, status, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      float* orow = out + static_cast<size_t>(row) * ldo;
      // forward_int8.rs:100-121: x + projected; residual may alias out.
      const float* rrow = residual ? residual + static_cast<size_t>(row) * ldo : nullptr;
      int32_t* arow = acc_out ? acc_out + static_cast<size_t>(row) * N : nullptr;
      // This warp's 32 x 32 staging block (16-byte chunks XOR-swizzled by row).
      float* stg = reinterpret_cast<float*>(smem + L::stg) + q * 32 * 32;
      const int row0 = m_blk * BM + q * 32;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32cols(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * acc_stride<BN>() + c * 32, v);
        const int col0 = n_blk * BN + c * 32;
        const float* sw = s_sw + c * 32;
        if (vec && !arow && col0 + 32 <= N && row0 + 32 <= M) {
          // Whole 32 x 32 block in range (warp-uniform): lane = row holds a
          // row's 32 columns; they go through shared memory so that each
          // store instruction writes four full 128-byte row segments instead
          // of 32 rows' 16 bytes.
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 w = *reinterpret_cast<const float4*>(sw + 4 * j);
            float4 o;
            o.x = rescale(static_cast<int>(v[4 * j]), s_a, w.x);
            o.y = rescale(static_cast<int>(v[4 * j + 1]), s_a, w.y);
            o.z = rescale(static_cast<int>(v[4 * j + 2]), s_a, w.z);
            o.w = rescale(static_cast<int>(v[4 * j + 3]), s_a, w.w);
            *reinterpret_cast<float4*>(stg + lane * 32 + 4 * (j ^ (lane & 7))) = o;
          }
          __syncwarp();
          const int rs = lane >> 3, jc = lane & 7;
          float4 o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + rs;
            o[i] = *reinterpret_cast<const float4*>(stg + r * 32 + 4 * (jc ^ (r & 7)));
          }
          __syncwarp();
          if (residual) {
            float4 rr[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              rr[i] = ld_act(reinterpret_cast<const float4*>(
                  residual + static_cast<size_t>(row0 + 4 * i + rs) * ldo + col0 + 4 * jc));
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              o[i].x = __fadd_rn(rr[i].x, o[i].x);
              o[i].y = __fadd_rn(rr[i].y, o[i].y);
              o[i].z = __fadd_rn(rr[i].z, o[i].z);
              o[i].w = __fadd_rn(rr[i].w, o[i].w);
            }
          }
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(out + static_cast<size_t>(row0 + 4 * i + rs) * ldo + col0 + 4 * jc) =
                o[i];
          // The other ranks' copies: whole 128-byte row segments over NVLink.
          for (int p = 0; p < go.ranks; ++p) {
            if (p == go.rank) continue;
            float* dst = go.stage[p] + ghalf + go.col0;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              *reinterpret_cast<float4*>(dst + static_cast<size_t>(row0 + 4 * i + rs) * ldo + col0 + 4 * jc) = o[i];
          }
          continue;
        }
        if (row < M) {
          if (vec && col0 + 32 <= N) {
            float4 r[8];
            if (rrow) {  // all residual loads in flight before the first use
#pragma unroll
              for (int j = 0; j < 8; ++j) r[j] = ld_act(reinterpret_cast<const float4*>(rrow + col0) + j);
            }
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 w = *reinterpret_cast<const float4*>(sw + j);
              float4 o;
              o.x = rescale(static_cast<int>(v[j]), s_a, w.x);
              o.y = rescale(static_cast<int>(v[j + 1]), s_a, w.y);
              o.z = rescale(static_cast<int>(v[j + 2]), s_a, w.z);
              o.w = rescale(static_cast<int>(v[j + 3]), s_a, w.w);
              if (rrow) {
                o.x = __fadd_rn(r[j / 4].x, o.x);
                o.y = __fadd_rn(r[j / 4].y, o.y);
                o.z = __fadd_rn(r[j / 4].z, o.z);
                o.w = __fadd_rn(r[j / 4].w, o.w);
              }
              *reinterpret_cast<float4*>(orow + col0 + j) = o;
              for (int p = 0; p < go.ranks; ++p)
                if (p != go.rank)
                  *reinterpret_cast<float4*>(go.stage[p] + ghalf + go.col0 + static_cast<size_t>(row) * ldo +
                                             col0 + j) = o;
              if (arow)
                *reinterpret_cast<int4*>(arow + col0 + j) =
                    make_int4(static_cast<int>(v[j]), static_cast<int>(v[j + 1]),
                              static_cast<int>(v[j + 2]), static_cast<int>(v[j + 3]));
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int col = col0 + j;
              if (col < N) {
                const float val = rescale(static_cast<int>(v[j]), s_a, sw[j]);
                orow[col] = rrow ? __fadd_rn(ld_act(rrow + col), val) : val;
                for (int p = 0; p < go.ranks; ++p)
                  if (p != go.rank) go.stage[p][ghalf + go.col0 + static_cast<size_t>(row) * ldo + col] = val;
                if (arow) arow[col] = static_cast<int>(v[j]);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
    if (go.ranks > 1) {
      // Gathered product: the CTA's tiles are on every rank; count the CTA in
      // on every rank's arrival counter.  Call state (go.seq, local): [0]
      // arrivals expected after the last call, [1] CTA ticket, [2] calls
      // issued (its parity picks the staging half).
      __threadfence_system();
      named_bar_sync(1, 32 * kEpiWarps);
      if (et == 0) {
        for (int p = 0; p < go.ranks; ++p) atomicAdd_system(go.ctr[p], 1ull);
        __threadfence();
        if (atomicAdd(go.seq + 1, 1ull) == gridDim.x - 1) {
          go.seq[1] = 0;
          go.seq[0] += static_cast<unsigned long long>(go.ranks) * gridDim.x;
          go.seq[2] = gseq + 1;
          __threadfence();
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kBufs * acc_stride<BN>())
                 : "memory");
  }
}

// ── 2-SM variant: tcgen05.mma.cta_group::2 over a CTA pair ─────────────────
// A cluster of two CTAs computes a 256 x BN tile: CTA r (rank in the pair)
// loads A rows [m0 + 128 r, +128) and the B rows [n0 + r BN/2, +BN/2) into its
// own shared memory, and the pair's even CTA issues one M = 256 MMA per K step
// that reads both CTAs' halves (each SM reads half of B; the 1-SM kernel reads
// all of B per SM, so a K step moves 26 KB per SM through shared memory
// instead of 36 KB at BN = 160).  D rows [128 r, +128) land in CTA r's TMEM;
// each CTA's epilogue drains its own 128 rows, as in the 1-SM kernel.
// Protocol (all waits bounded):
//   full[s]   (even CTA) : one arrival with the pair's bytes; both CTAs' TMA
//                          loads complete their bytes there (its address
//                          taken with mapa in the odd CTA);
//   empty[s]  (each CTA) : the MMA thread's commit, arriving on the barrier at
//                          the same offset in both CTAs (CTA mask 0b11);
//   tfull[b]  (each CTA) : likewise, once a tile's MMAs are done;
//   tempty[b] (even CTA) : 2 x 4 epilogue-warp arrivals (remote from the odd
//                          CTA) before the MMAs reuse accumulator buffer b.
// TMEM is allocated and freed with cta_group::2 by warp 1 of both CTAs; a
// cluster barrier follows barrier initialisation and precedes the free, so
// neither CTA's shared memory or TMEM goes away while the other uses it.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* tm, int x, int y,
                                                 uint32_t bar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar_cluster_addr)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster_addr)
               : "memory");
}
// The same commit arriving on the barrier at this shared-memory offset in both
// CTAs of the pair (CTA mask 0b11): one instruction instead of two.
__device__ __forceinline__ void umma_commit_both(const uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_addr(bar))
      : "memory");
}
// kind::i8 instruction descriptor for the pair's M = 256.
template <int BN>
__device__ __forceinline__ uint32_t idesc_i8_pair() {
  return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(256 >> 4) << 24);
}

template <int BN, int kStages>
struct Tc2Layout {
  static constexpr size_t a_bytes = BM * BK;
  static constexpr size_t b_bytes = (BN / 2) * BK;
  static constexpr size_t stage_bytes = a_bytes + b_bytes;
  static constexpr size_t epi = kStages * stage_bytes;
  static constexpr size_t epi_bytes = 2 * 256 * 4;
  static constexpr size_t stg = epi + epi_bytes;
  static constexpr size_t bars = stg + kStgBytes;
  // full[S], empty[S], tfull[2], tempty[2], sready[2], mma_done, abort flag + tmem slot
  static constexpr size_t bars_bytes = (2 * kStages + 7) * 8 + 16;
  static constexpr size_t total = bars + bars_bytes + 1024;
};

template <int BN, int kStages>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    gemm_i8_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const float* __restrict__ act_scale, int scale_per_row,
                       const float* __restrict__ w_scales, const __grid_constant__ GemmOut go, int M, int N,
                       int K, int* status) {
  using L = Tc2Layout<BN, kStages>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bars);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* sready = tempty + 2;
  uint64_t* mma_done = sready + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(mma_done + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1) + 1;
  float* const out = go.out;
  const size_t ldo = go.ldo;

  const uint32_t rank = cluster_rank();  // 0: the pair's MMA issuer
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + 2 * BM - 1) / (2 * BM), n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kEpiWarps);
      mbar_init(&sready[b], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(2 * acc_stride<BN>())
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
      const int my_tiles = pair < num_tiles ? (num_tiles - 1 - pair) / n_pairs + 1 : 0;
      const int iters = my_tiles * kblocks;
      const int pre = std::min(kStages, iters);
      // The even CTA's full barriers, addressed from either CTA.
      const uint32_t full0 = mapa_shared(smem_addr(full), 0);
      auto full_at = [&](int s) { return full0 + static_cast<uint32_t>(s) * 8u; };
      for (int it = 0; it < pre; ++it) {
        const int tile = pair + (it / kblocks) * n_pairs, kb = it % kblocks;
        uint8_t* sa = smem + it * L::stage_bytes;
        if (rank == 0) mbar_arrive_expect_tx(&full[it], static_cast<uint32_t>(2 * L::stage_bytes));
        tma_load_2d_pair(sa + L::a_bytes, &tmB, kb * BK, (tile / m_tiles) * BN + static_cast<int>(rank) * (BN / 2),
                         full_at(it));
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int it = 0; it < pre; ++it) {
        const int tile = pair + (it / kblocks) * n_pairs, kb = it % kblocks;
        tma_load_2d_pair(smem + it * L::stage_bytes, &tmA, kb * BK,
                         (tile % m_tiles) * 2 * BM + static_cast<int>(rank) * BM, full_at(it));
      }
      int it = pre;
      for (; it < iters; ++it) {
        const int s = it % kStages;
        if (!wait_or_abort(&empty[s], ((it / kStages) - 1) & 1, status, abort_flag)) break;
        const int tile = pair + (it / kblocks) * n_pairs, kb = it % kblocks;
        uint8_t* sa = smem + s * L::stage_bytes;
        if (rank == 0) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(2 * L::stage_bytes));
        tma_load_2d_pair(sa, &tmA, kb * BK, (tile % m_tiles) * 2 * BM + static_cast<int>(rank) * BM, full_at(s));
        tma_load_2d_pair(sa + L::a_bytes, &tmB, kb * BK, (tile / m_tiles) * BN + static_cast<int>(rank) * (BN / 2),
                         full_at(s));
      }
      // Drain: the even CTA waits for every phase it expected (both CTAs'
      // bytes).  The odd CTA cannot wait on those barriers; its copies landed
      // before the even CTA's waits on them completed, which the final
      // cluster barrier orders before either CTA exits.  After an abort it
      // gives its copies in flight a bounded moment instead.
      if (rank == 0) {
        for (int j = std::max(0, it - kStages); j < it; ++j)
          mbar_wait(&full[j % kStages], (j / kStages) & 1, status);
      } else if (*abort_flag) {
        __nanosleep(1000000);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = idesc_i8_pair<BN>();
      int it = 0, t = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += n_pairs, ++t) {
        const int b = t & 1;
        if (t >= 2 && !wait_or_abort(&tempty[b], ((t >> 1) - 1) & 1, status, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * acc_stride<BN>();
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!wait_or_abort(&full[s], (it / kStages) & 1, status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* sa = smem + s * L::stage_bytes;
          const uint64_t adesc = smem_desc_sw128(sa);
          const uint64_t bdesc = smem_desc_sw128(sa + L::a_bytes);
#pragma unroll
          for (int j = 0; j < BK / UMMA_K; ++j)
            umma_i8_pair(d_tmem, adesc + 2 * j, bdesc + 2 * j, idesc, (kb | j) != 0);
          umma_commit_both(&empty[s]);
        }
        if (ok) umma_commit_both(&tfull[b]);
      }
      // All MMAs issued by this thread are complete before TMEM is freed.
      umma_commit_pair(smem_addr(mma_done));
      mbar_wait(mma_done, 0, status);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int et = threadIdx.x - 64;  // 0..127 among the epilogue warps
    const uint32_t tempty0 = mapa_shared(smem_addr(tempty), 0);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const float s_all = scale_per_row ? 0.0f : ld_act(act_scale);
    const bool vec = (N % 4) == 0 && (ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                     (go.ranks <= 1 || (go.col0 % 4) == 0);
    const unsigned long long gseq = go.ranks > 1 ? ld_act(go.seq + 2) : 0ull;
    const size_t ghalf = (gseq & 1) * go.half;
    int t = 0;
    for (int tile = pair; tile < num_tiles; tile += n_pairs, ++t) {
      const int b = t & 1;
      const int m_blk = tile % m_tiles, n_blk = tile / m_tiles;
      const int row0 = m_blk * 2 * BM + static_cast<int>(rank) * BM + q * 32;
      const int row = row0 + lane;
      float* s_sw = reinterpret_cast<float*>(smem + L::epi) + b * 256;
      for (int i = et; i < BN; i += 32 * kEpiWarps) {
        const int col = n_blk * BN + i;
        s_sw[i] = col < N ? __ldg(w_scales + col) : 0.0f;
      }
      const float s_a = scale_per_row ? (row < M ? ld_act(act_scale + row) : 0.0f) : s_all;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sready[b]);
      bool ok = wait_or_abort(&sready[b], (t >> 1) & 1, status, abort_flag);
      ok = ok && wait_or_abort(&tfull[b], (t >> 1) & 1, status, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      float* orow = out + static_cast<size_t>(row) * ldo;
      float* stg = reinterpret_cast<float*>(smem + L::stg) + q * 32 * 32;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32cols(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * acc_stride<BN>() + c * 32, v);
        const int col0 = n_blk * BN + c * 32;
        const float* sw = s_sw + c * 32;
        if (vec && col0 + 32 <= N && row0 + 32 <= M) {
          // Whole 32 x 32 block in range: staged through shared memory so
          // each store instruction writes four full 128-byte row segments.
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 w = *reinterpret_cast<const float4*>(sw + 4 * j);
            float4 o;
            o.x = rescale(static_cast<int>(v[4 * j]), s_a, w.x);
            o.y = rescale(static_cast<int>(v[4 * j + 1]), s_a, w.y);
            o.z = rescale(static_cast<int>(v[4 * j + 2]), s_a, w.z);
            o.w = rescale(static_cast<int>(v[4 * j + 3]), s_a, w.w);
            *reinterpret_cast<float4*>(stg + lane * 32 + 4 * (j ^ (lane & 7))) = o;
          }
          __syncwarp();
          const int rs = lane >> 3, jc = lane & 7;
          float4 o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + rs;
            o[i] = *reinterpret_cast<const float4*>(stg + r * 32 + 4 * (jc ^ (r & 7)));
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(out + static_cast<size_t>(row0 + 4 * i + rs) * ldo + col0 + 4 * jc) = o[i];
          for (int p = 0; p < go.ranks; ++p) {
            if (p == go.rank) continue;
            float* dst = go.stage[p] + ghalf + go.col0;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              *reinterpret_cast<float4*>(dst + static_cast<size_t>(row0 + 4 * i + rs) * ldo + col0 + 4 * jc) = o[i];
          }
          continue;
        }
        if (row < M) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = col0 + j;
            if (col < N) {
              const float val = rescale(static_cast<int>(v[j]), s_a, sw[j]);
              orow[col] = val;
              for (int p = 0; p < go.ranks; ++p)
                if (p != go.rank) go.stage[p][ghalf + go.col0 + static_cast<size_t>(row) * ldo + col] = val;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&tempty[b]);
        else
          mbar_arrive_cluster(tempty0 + static_cast<uint32_t>(b) * 8u);
      }
    }
    if (go.ranks > 1) {
      __threadfence_system();
      named_bar_sync(1, 32 * kEpiWarps);
      if (et == 0) {
        for (int p = 0; p < go.ranks; ++p) atomicAdd_system(go.ctr[p], 1ull);
        __threadfence();
        if (atomicAdd(go.seq + 1, 1ull) == gridDim.x - 1) {
          go.seq[1] = 0;
          go.seq[0] += static_cast<unsigned long long>(go.ranks) * gridDim.x;
          go.seq[2] = gseq + 1;
          __threadfence();
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the even CTA's MMAs no longer read the odd CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(2 * acc_stride<BN>())
                 : "memory");
  }
}

// ── host side ────────────────────────────────────────────────────────────────

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_map(CUtensorMap* tm, const void* base, size_t rows, size_t k, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename KernelT>
cudaError_t set_smem_tc(KernelT k, size_t bytes, int device) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(reinterpret_cast<const void*>(k), device);
  auto it = done.find(key);
  if (it != done.end() && bytes <= it->second) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(bytes));
  if (e == cudaSuccess) done[key] = bytes;
  return e;
}

// Tile width: the BN (a multiple of 32 from 128 to 256; tcgen05 needs N % 16
// == 0 at M = 128, the epilogue reads 32 TMEM columns at a time) that
// minimises rounds-of-tiles x BN over the persistent grid, larger BN on ties
// (fewer shared-memory bytes per MMA).  The context's MRI_OPT_GEMM_BN forces one.
int pick_bn(const DeviceInfo& dev, size_t M, size_t N) {
  const int v = dev.opt.gemm_bn;
  if (v >= 128 && v <= 256 && v % 32 == 0) return v;
  const size_t mt = (M + BM - 1) / BM;
  int best = 128;
  size_t best_cost = ~size_t(0);
  for (int bn = 256; bn >= 128; bn -= 32) {
    const size_t tiles = mt * ((N + bn - 1) / bn);
    const size_t cost = ((tiles + dev.sm_count - 1) / dev.sm_count) * bn;
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

template <int BN, int kStages, int kBufs = 2>
cudaError_t launch_bn(const DeviceInfo& dev, cudaStream_t st, const CUtensorMap& ta,
                      const CUtensorMap& tb, const float* act_scale, int per_row,
                      const float* w_scales, size_t M, size_t N, size_t K, const GemmOut& out,
                      int32_t* acc_out, int* status, const float* residual, int grid) {
  static_assert(TcLayout<BN, kStages, kBufs>::total <= 232448,
                "stage ring exceeds the per-CTA shared memory");
  // Two CTAs per SM: both rings plus the 1 KB the runtime reserves per CTA
  // within the SM's 228 KB.
  static_assert(kBufs == 2 || 2 * (TcLayout<BN, kStages, kBufs>::total + 1024) <= 233472,
                "two CTAs per SM do not fit");
  const size_t smem = TcLayout<BN, kStages, kBufs>::total;
  cudaError_t e = set_smem_tc(gemm_i8_tc_kernel<BN, kStages, kBufs>, smem, dev.device);
  if (e != cudaSuccess) return e;
  const size_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  // One tile per CTA when kBufs == 1; a persistent grid otherwise.
  if (grid < 1 || (kBufs == 1 && static_cast<size_t>(grid) != tiles)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dev.opt.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemm_i8_tc_kernel<BN, kStages, kBufs>, ta, tb, act_scale, per_row, w_scales,
                            out, acc_out, static_cast<int>(M), static_cast<int>(N),
                            static_cast<int>(K), status, residual);
}

template <int BN, int kStages>
cudaError_t launch_pair(const DeviceInfo& dev, cudaStream_t st, const CUtensorMap& ta, const CUtensorMap& tb,
                        const float* act_scale, int per_row, const float* w_scales, size_t M, size_t N, size_t K,
                        const GemmOut& out, int* status, int grid) {
  static_assert(Tc2Layout<BN, kStages>::total <= 232448, "stage ring exceeds the per-CTA shared memory");
  static_assert(BN % 32 == 0 && BN >= 128 && BN <= 256, "a cta_group::2 M = 256 kind::i8 MMA needs N % 32 == 0");
  const size_t smem = Tc2Layout<BN, kStages>::total;
  cudaError_t e = set_smem_tc(gemm_i8_tc2_kernel<BN, kStages>, smem, dev.device);
  if (e != cudaSuccess) return e;
  if (grid < 2 || grid % 2) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dev.opt.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemm_i8_tc2_kernel<BN, kStages>, ta, tb, act_scale, per_row, w_scales, out,
                            static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), status);
}

}  // namespace

bool gemm_i8_tc_supported(const DeviceInfo& dev, size_t M, size_t N, size_t K) {
  if (dev.cc_major != 10) return false;
  if (M < 1 || N < 1 || K < 16 || K % 16 != 0) return false;
  if (M > (1u << 30) || N > (1u << 30) || K > (1u << 30)) return false;
  return encode_fn() != nullptr;
}

// Ring stages of the pair kernel (26-32 KB per stage and CTA).
static int pair_stages(int bn) { return bn <= 160 ? 7 : (bn <= 192 ? 6 : 5); }

// Stage counts keep the ring within the 227 KB a CTA may use.
static int persistent_stages(int bn) {
  switch (bn) {
    case 128: return 6;
    case 160: return 5;
    case 192: return 5;
    case 224: return 4;
    default: return 4;
  }
}

// Tile width of the pair kernel: the BN (128..256 step 32, a valid N of a
// cta_group::2 M = 256 MMA) minimising rounds-of-pair-tiles x BN over the
// CTA pairs, larger on ties.
static int pick_bn_pair(int pairs, size_t M, size_t N) {
  const size_t mt = (M + 2 * BM - 1) / (2 * BM);
  int best = 128;
  size_t best_cost = ~size_t(0);
  for (int bn = 256; bn >= 128; bn -= 32) {
    const size_t tiles = mt * ((N + bn - 1) / bn);
    const size_t cost = ((tiles + pairs - 1) / pairs) * bn;
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

cudaError_t gemm_i8_tc_plan(const DeviceInfo& dev, size_t M, size_t N, size_t K, GemmPlan* plan, bool plain) {
  if (!gemm_i8_tc_supported(dev, M, N, K)) return cudaErrorInvalidValue;
  GemmPlan p;
  // SMs the grid may use (an internal reserve can keep some free).
  const int sms = std::max(2, dev.sm_count - std::max(0, dev.opt.sm_reserve));
  // CTA pairs (M = 256 MMAs, each SM reading half of the weight tile) for
  // plain outputs from four rounds of pair tiles on: measured 2.55 against
  // 2.40 POPS at [2048, 8192] x [8192, 28672] (19.5 rounds), but 30.1 against
  // 23.0 us at the [512, 4096] x [4096, 11008] prefill shape (1.9 rounds),
  // where the pair's fixed cost per call (cluster set-up, the last tile's
  // exposed epilogue on one CTA per SM) is not amortised.  MRI_OPT_GEMM_PAIR =
  // 2 takes pairs for any plain output of more than 128 rows (tests).
  const int pairs = sms / 2;
  const int bn_pair = dev.opt.gemm_bn ? dev.opt.gemm_bn : pick_bn_pair(pairs, M, N);
  const size_t pair_tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + bn_pair - 1) / bn_pair);
  const bool use_pair = plain && M > BM &&
                        (dev.opt.gemm_pair == 2 ||
                         (dev.opt.gemm_pair == 1 && pair_tiles >= 4 * static_cast<size_t>(pairs)));
  if (use_pair) {
    const int bn = bn_pair;
    p.pair = 2;
    p.bn = bn;
    p.tiles = static_cast<int>(((M + 2 * BM - 1) / (2 * BM)) * ((N + bn - 1) / bn));
    p.bufs = 2;
    p.stages = pair_stages(bn);
    p.grid = 2 * std::min(p.tiles, pairs);
    p.tiles_per_cta = (p.tiles + p.grid / 2 - 1) / (p.grid / 2);
    *plan = p;
    return cudaSuccess;
  }
  DeviceInfo d2 = dev;
  d2.sm_count = sms;
  p.bn = pick_bn(d2, M, N);
  p.tiles = static_cast<int>(((M + BM - 1) / BM) * ((N + p.bn - 1) / p.bn));
  // Between one and two rounds of tiles, one tile per CTA with two CTAs per
  // SM (3-stage rings, one accumulator buffer each): the second CTA's loads
  // and MMAs fill the first one's gaps, and each CTA's epilogue overlaps the
  // other's main loop.  The context's MRI_OPT_GEMM_2CTA = 0 keeps the
  // persistent grid.
  if (dev.opt.gemm_2cta && (p.bn == 128 || p.bn == 160) && p.tiles > sms && p.tiles <= 2 * sms) {
    p.bufs = 1;
    p.stages = 3;
    p.grid = p.tiles;
  } else {
    p.bufs = 2;
    p.stages = persistent_stages(p.bn);
    p.grid = std::min(p.tiles, sms);
  }
  p.tiles_per_cta = (p.tiles + p.grid - 1) / p.grid;
  *plan = p;
  return cudaSuccess;
}

cudaError_t launch_gemm_i8_tc(const DeviceInfo& dev, cudaStream_t st, const int8_t* xq,
                              const float* act_scale_dev, int scale_per_row, const int8_t* W,
                              const float* w_scales, size_t M, size_t N, size_t K, float* out_ptr,
                              int32_t* acc_out, int* status, LaunchStats* ls,
                              const float* residual, const GemmOut* gather) {
  if ((reinterpret_cast<uintptr_t>(xq) & 15) || (reinterpret_cast<uintptr_t>(W) & 15))
    return cudaErrorMisalignedAddress;
  GemmOut out;
  if (gather) {
    if (gather->ranks < 2 || gather->ranks > EpiArgs::kMaxRanks || residual || acc_out || !gather->seq)
      return cudaErrorInvalidValue;
    out = *gather;
  } else {
    out.out = out_ptr;
    out.ldo = N;
  }
  GemmPlan p;
  if (cudaError_t e = gemm_i8_tc_plan(dev, M, N, K, &p, !residual && !acc_out)) return e;
  CUtensorMap ta, tb;
  if (!make_map(&ta, xq, M, K, BM) || !make_map(&tb, W, N, K, p.pair == 2 ? p.bn / 2 : p.bn))
    return cudaErrorInvalidValue;
  cudaError_t e;
  if (p.pair == 2) {
#define MRI_GEMM2_CASE(BNV)                                                                                     \
  case BNV:                                                                                                   \
    e = launch_pair<BNV, (BNV <= 160 ? 7 : (BNV <= 192 ? 6 : 5))>(dev, st, ta, tb, act_scale_dev, scale_per_row,  \
                                               w_scales, M, N, K, out, status, p.grid);                        \
    break;
    switch (p.bn) {
      MRI_GEMM2_CASE(128)
      MRI_GEMM2_CASE(160)
      MRI_GEMM2_CASE(192)
      MRI_GEMM2_CASE(224)
      MRI_GEMM2_CASE(256)
      default: e = cudaErrorInvalidValue;
    }
#undef MRI_GEMM2_CASE
    if (ls) ls->launches++;
    return e;
  }
#define MRI_GEMM_ARGS dev, st, ta, tb, act_scale_dev, scale_per_row, w_scales, M, N, K, out, acc_out, status, residual, p.grid
  if (p.bufs == 1) {
    e = p.bn == 128 ? launch_bn<128, 3, 1>(MRI_GEMM_ARGS) : launch_bn<160, 3, 1>(MRI_GEMM_ARGS);
  } else {
    switch (p.bn) {
      case 128: e = launch_bn<128, 6>(MRI_GEMM_ARGS); break;
      case 160: e = launch_bn<160, 5>(MRI_GEMM_ARGS); break;
      case 192: e = launch_bn<192, 5>(MRI_GEMM_ARGS); break;
      case 224: e = launch_bn<224, 4>(MRI_GEMM_ARGS); break;
      default: e = launch_bn<256, 4>(MRI_GEMM_ARGS);
    }
  }
#undef MRI_GEMM_ARGS
  if (ls) ls->launches++;
  return e;
}

}  // namespace mri
