"""Every kernel variant the benchmarks run, pinned to the oracle at the
benchmarked shapes (INT8 bars: INT32 sums and f32 outputs bit-exact).

Each test first asks the library which launch shape it will use for the shape
(mri_int8_gemm_plan / mri_int8_gemv_plan) and asserts that it is the variant
the test is meant to cover, so a change of dispatch cannot silently move a
benchmarked path out from under its test.  The oracle here is
matmul_int8_parallel (parallel.rs:308-346) with its INT32 sums, which equals
the scalar matmul_int8 (int8.rs:61-98) element for element and finishes
these sizes in seconds on the host's cores.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def weights(rng, n, k):
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    return wq, ws


def oracle_from_f32(oracle, x, wq, ws, n, k):
    """matmul_int8_from_f32 (int8.rs:113-143) as proj_int8_par runs it
    (forward_int8.rs:87-96): per-tensor quantize_symmetric, then the
    row-parallel product; returns (out, acc)."""
    m = x.shape[0]
    aq, s = oracle.quantize_symmetric(x)
    acc = np.empty((m, n), np.int32)
    out = oracle.matmul_int8_parallel(aq, s, wq, ws, n, k, m, acc_out=acc)
    return out, acc, aq, s


def check_prequantized(mri, oracle, aq, s, wq, ws, qm, m, n, k):
    """matmul_int8 with the INT32 sums requested (direct-store epilogue)."""
    acc = np.zeros((m, n), np.int32)
    got = mri.matmul_int8(aq, s, qm, m, acc_out=acc)
    want_acc = np.empty((m, n), np.int32)
    want = oracle.matmul_int8_parallel(aq, s, wq, ws, n, k, m, acc_out=want_acc)
    assert np.array_equal(acc, want_acc), f"{np.count_nonzero(acc != want_acc)} INT32 sums differ"
    assert np.array_equal(bits(got), bits(want))


# ── tensor-core GEMM ─────────────────────────────────────────────────────────

# (m, n, k, fewest tiles per CTA): the 7B prefill gate/up GEMM at 1024 rows
# (4 tiles per CTA: each TMEM buffer is reused, so its waits on the
# epilogue's release run), and a Llama-70B gate/up shard of an 8-GPU node at
# 2048 rows (N = 28672 / 8).
PERSISTENT_SHAPES = [(1024, 11008, 4096, 3), (2048, 3584, 8192, 2)]


@pytest.mark.parametrize("m,n,k,min_tiles", PERSISTENT_SHAPES)
def test_gemm_persistent_multi_tile_exact(mri, oracle, gpu_ctx, ctx_option, m, n, k, min_tiles):
    """The one-CTA persistent grid (OPT_GEMM_PAIR = 0) with two TMEM
    accumulator buffers and several tiles per CTA (tile t + 1's MMAs run while
    tile t drains; from the third tile on a buffer waits for the epilogue's
    release).  Every row, both epilogues: the staged f32 stores (no INT32
    copy) through matmul_int8_from_f32, and the direct stores with INT32
    sums."""
    ctx_option(mri.OPT_GEMM_PAIR, 0)
    plan = gpu_ctx.int8_gemm_plan(m, n, k)
    assert plan["cta_pair"] == 1 and plan["acc_buffers"] == 2 and plan["tiles_per_cta"] >= min_tiles, plan
    assert plan["grid"] <= 148, plan
    rng = np.random.default_rng(m + n)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wq, ws = weights(rng, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    want, want_acc, aq, s = oracle_from_f32(oracle, x, wq, ws, n, k)
    got = mri.matmul_int8_from_f32(x, qm)
    assert np.array_equal(bits(got), bits(want)), f"{np.count_nonzero(bits(got) != bits(want))} outputs differ"
    acc = np.zeros((m, n), np.int32)
    got = mri.matmul_int8(aq, s, qm, m, acc_out=acc)
    assert np.array_equal(acc, want_acc)
    assert np.array_equal(bits(got), bits(want))


def test_gemm_persistent_grid_when_two_cta_off(mri, oracle, gpu_ctx, ctx_option):
    """OPT_GEMM_2CTA = 0 between one and two rounds of tiles (the prefill
    shape, 276 tiles): the persistent grid, two tiles on most CTAs, every
    row against the oracle."""
    m, n, k = 512, 11008, 4096
    ctx_option(mri.OPT_GEMM_PAIR, 0)
    assert gpu_ctx.int8_gemm_plan(m, n, k)["acc_buffers"] == 1
    ctx_option(mri.OPT_GEMM_2CTA, 0)
    plan = gpu_ctx.int8_gemm_plan(m, n, k)
    assert plan["acc_buffers"] == 2 and plan["tiles_per_cta"] == 2 and plan["grid"] == 148, plan
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wq, ws = weights(rng, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    want, want_acc, aq, s = oracle_from_f32(oracle, x, wq, ws, n, k)
    assert np.array_equal(bits(mri.matmul_int8_from_f32(x, qm)), bits(want))
    acc = np.zeros((m, n), np.int32)
    got = mri.matmul_int8(aq, s, qm, m, acc_out=acc)
    assert np.array_equal(acc, want_acc)
    assert np.array_equal(bits(got), bits(want))


# (m, n, k): ragged rows and columns, one pair tile, several tiles per pair
# (a 70B gate/up shard of an 8-GPU node at 2048 rows), the 7B gate/up at 1024
# rows, and the full 70B gate/up at 2048 rows (19.5 rounds of pair tiles: the
# default takes pairs there).
PAIR_SHAPES = [(129, 1000, 256), (300, 520, 4352), (256, 160, 128), (2048, 3584, 8192), (1024, 11008, 4096),
               (2048, 28672, 8192)]


@pytest.mark.parametrize("m,n,k", PAIR_SHAPES)
def test_gemm_cta_pair_exact(mri, oracle, gpu_ctx, ctx_option, m, n, k):
    """The CTA-pair kernel: each CTA of a two-CTA cluster loads its 128 rows
    of activations and half of the weight tile, the even CTA issues M = 256
    MMAs over both, each CTA drains its TMEM rows.  Every output against the
    oracle, on two calls in a row (barrier phases and TMEM buffers reused).
    OPT_GEMM_PAIR = 2 takes pairs at every size (by default they run from
    four rounds of pair tiles on)."""
    ctx_option(mri.OPT_GEMM_PAIR, 2)
    plan = gpu_ctx.int8_gemm_plan(m, n, k)
    assert plan["cta_pair"] == 2, plan
    rng = np.random.default_rng(m * 3 + n)
    wq, ws = weights(rng, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    for rep in range(2):
        x = rng.normal(0, 1 + rep, size=(m, k)).astype(np.float32)
        want, _, _, _ = oracle_from_f32(oracle, x, wq, ws, n, k)
        got = mri.matmul_int8_from_f32(x, qm)
        assert np.array_equal(bits(got), bits(want)), (rep, int(np.count_nonzero(bits(got) != bits(want))))


@pytest.fixture(scope="module")
def prefill_case(mri, oracle):
    """BASELINE prefill config: A from N(0,1) activations [512, 4096], B the
    per-channel quantization of N(0, 0.02) weights [11008, 4096]; seed 1."""
    rng = np.random.default_rng(1)
    m, n, k = 512, 11008, 4096
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wf = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    wq, ws = oracle.quantize_per_channel(wf, n, k)
    return x, wq, ws, m, n, k


@pytest.mark.parametrize("pair", [2, 0], ids=["cta_pair", "one_cta"])
def test_prefill_all_rows_per_tensor(mri, oracle, gpu_ctx, ctx_option, prefill_case, pair):
    """matmul_int8_from_f32 at the prefill config, on the one-CTA kernel (the
    default here: two CTAs per SM, one tile each) and on the CTA-pair kernel
    (OPT_GEMM_PAIR = 2: 256-row tiles, tcgen05.mma.cta_group::2): all 512 x
    11008 outputs bit-equal to the oracle, and all INT32 sums through
    matmul_int8."""
    x, wq, ws, m, n, k = prefill_case
    ctx_option(mri.OPT_GEMM_PAIR, pair)
    plan = gpu_ctx.int8_gemm_plan(m, n, k)
    if pair:
        assert plan["cta_pair"] == 2 and plan["grid"] % 2 == 0, plan
    else:
        assert plan["cta_pair"] == 1 and plan["acc_buffers"] == 1 and plan["grid"] == plan["tiles"], plan
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    want, want_acc, aq, s = oracle_from_f32(oracle, x, wq, ws, n, k)
    assert np.array_equal(bits(mri.matmul_int8_from_f32(x, qm)), bits(want))
    check_prequantized(mri, oracle, aq, s, wq, ws, qm, m, n, k)


def test_prefill_all_rows_per_row(mri, oracle, gpu_ctx, prefill_case):
    """The per-row granularity BASELINE's prefill config names (each
    activation row quantized with its own scale, q8_direct.rs:260-264), all
    rows: out[m, n] = ((f32)acc * s_a[m]) * s_w[n] with the oracle's sums
    and per-row scales."""
    x, wq, ws, m, n, k = prefill_case
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    got = mri.matmul_int8_from_f32(x, qm, granularity=mri.PER_ROW)
    aq, sr = oracle.quantize_symmetric_rows(x, m, k)
    acc = np.empty((m, n), np.int32)
    oracle.matmul_int8_parallel(aq, np.float32(1.0), wq, ws, n, k, m, acc_out=acc)
    want = (acc.astype(np.float32) * sr[:, None]).astype(np.float32) * ws[None, :]
    assert np.array_equal(bits(got), bits(want))


# ── streaming GEMV at the benchmarked long-K shapes ──────────────────────────

# (m, n, k): the 7B down projection (K = 11008) at 1 and 8 rows, the 70B down
# projection (K = 28672) at 1 row, and the 70B gate/up (K = 8192).
GEMV_SHAPES = [(1, 4096, 11008), (8, 4096, 11008), (1, 8192, 28672), (1, 28672, 8192)]


def test_70b_down_projection_at_8_rows_takes_the_gemm(mri, oracle, gpu_ctx):
    """8 rows of K = 28672 do not fit the streaming GEMV's shared-memory
    activations; the product runs on the tensor-core GEMM (one 128-row tile
    row, rows 8..127 zero-filled by TMA) and matches the oracle."""
    m, n, k = 8, 8192, 28672
    assert gpu_ctx.int8_path(m, n, k) == 2
    rng = np.random.default_rng(828)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wq, ws = weights(rng, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    want, _, aq, s = oracle_from_f32(oracle, x, wq, ws, n, k)
    assert np.array_equal(bits(mri.matmul_int8_from_f32(x, qm)), bits(want))
    check_prequantized(mri, oracle, aq, s, wq, ws, qm, m, n, k)


@pytest.mark.parametrize("m,n,k", GEMV_SHAPES)
def test_gemv_long_k_exact(mri, oracle, gpu_ctx, m, n, k):
    """The streaming INT8 GEMV with K-chunked stages: the register prologue
    (width 12) where the input fits it, else the quantize-first path (the
    quantizer kernels, then int8 activations streamed with the device scale).
    f32 input through matmul_int8_from_f32, and pre-quantized input with the
    INT32 sums, against the oracle."""
    assert gpu_ctx.int8_path(m, n, k) == 0
    plan = gpu_ctx.int8_gemv_plan(m, n, k)
    assert plan["grid"] <= plan["ctas_per_sm"] * 148, plan
    assert plan["ctas_per_sm"] <= plan["resident_ctas"], plan
    if k >= 11008:
        assert plan["k_chunks"] > 1, plan
    if (m, k) == (1, 11008):
        assert plan["reg_vec"] == 12 and plan["quantize_first"] == 0, plan
    if k == 28672 or m == 8:
        assert plan["reg_vec"] == 0 and plan["quantize_first"] == 1, plan
    if (m, k) == (1, 8192):
        assert plan["reg_vec"] == 12, plan
    rng = np.random.default_rng(m * 7 + k)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wq, ws = weights(rng, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    want, _, aq, s = oracle_from_f32(oracle, x, wq, ws, n, k)
    assert np.array_equal(bits(mri.matmul_int8_from_f32(x, qm)), bits(want))
    check_prequantized(mri, oracle, aq, s, wq, ws, qm, m, n, k)


def test_pdl_off_same_results(mri, oracle, ctx_option):
    """OPT_PDL = 0 (every kernel launched without programmatic dependent
    launch): the decode GEMV and the prefill GEMM give the oracle's outputs."""
    ctx_option(mri.OPT_PDL, 0)
    rng = np.random.default_rng(77)
    for m, n, k in ((1, 11008, 4096), (300, 2000, 4096)):
        x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
        wq, ws = weights(rng, n, k)
        want, _, _, _ = oracle_from_f32(oracle, x, wq, ws, n, k)
        got = mri.matmul_int8_from_f32(x, mri.QuantizedMatrix(wq, ws, n, k))
        assert np.array_equal(bits(got), bits(want))


# ── Q8_0 / Q4_0 at 2..8 rows without the warp-MMA kernels ────────────────────

@pytest.mark.parametrize("m", [2, 8])
def test_q8_0_streaming_kernel_when_mma_off(mri, oracle, ctx_option, m):
    """OPT_Q8_MMA = 0: Q8_0 at m = 2..8 on the streaming kernel (per-row
    quantization in its prologue, dp4a block dots), bit-exact."""
    ctx_option(mri.OPT_Q8_MMA, 0)
    rng = np.random.default_rng(30 + m)
    n, k = 2048, 4096
    wb = oracle.quantize_q8_0_matrix(rng.normal(0, 0.02, size=(n, k)).astype(np.float32), n, k)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    got = mri.matmul_q8_0_direct(x, mri.Q8_0WeightMatrix.from_raw_bytes(wb, n, k))
    want = oracle.matmul_q8_0_direct(x, m, k, wb, n, k)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("m", [2, 8])
def test_q4_0_streaming_kernel_when_mma_off(mri, oracle, ctx_option, m):
    """OPT_Q4_MMA = 0: Q4_0 at m = 2..8 on the CUDA-core streaming kernel,
    within 1e-3 relative (absolute floor 1e-5 * sum |x * w|)."""
    from test_gpu_parity import q4_close
    ctx_option(mri.OPT_Q4_MMA, 0)
    rng = np.random.default_rng(40 + m)
    n, k = 2048, 4096
    wb = oracle.quantize_q4_0_matrix(rng.normal(0, 0.02, size=(n, k)).astype(np.float32), n, k)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    got = mri.matmul_q4_0_dequant(x, wb, n, k)
    want = oracle.matmul_q4_0_dequant(x, m, k, wb, n, k)
    ok, worst = q4_close(got, want, x, oracle.dequantize_q4_0(wb).reshape(n, k))
    assert ok, worst


def test_options_reject_bad_values(mri, gpu_ctx):
    with pytest.raises(ValueError):
        gpu_ctx.set_option(mri.OPT_GEMM_BN, 100)
    with pytest.raises(ValueError):
        gpu_ctx.set_option(99, 1)
    assert gpu_ctx.get_option(mri.OPT_PDL) == 1


# ── the one-launch per-tensor quantizer ──────────────────────────────────────

@pytest.mark.parametrize("m,k", [(1, 16), (1, 28672), (512, 4096), (2048, 8192), (3, 4100), (7, 5)])
def test_one_launch_quantizer_repeated_calls_exact(mri, oracle, gpu_ctx, m, k):
    """quantize_symmetric per tensor (symmetric.rs:42-57) through the
    one-launch kernel (grid barrier between the absmax and the quantization;
    at 2048 x 8192 most values are re-read after the barrier, at 512 x 4096
    all stay in registers) and, for sizes not a multiple of 4, the two-kernel
    path: scale and codes bit-equal to the oracle on three calls in a row
    with different inputs (the barrier words are reused)."""
    import torch
    rng = np.random.default_rng(m + k)
    q = torch.empty(m, k, dtype=torch.int8, device="cuda")
    s = torch.empty(1, device="cuda")
    lib = mri._lib.load()
    for rep in range(3):
        x = (rng.normal(0, 1, size=(m, k)) * (1.0 + 3 * rep)).astype(np.float32)
        x.reshape(-1)[rng.integers(0, m * k)] = 0.5 * np.abs(x).max()
        xd = torch.from_numpy(x).cuda()
        torch.cuda.synchronize()
        rc = lib.mri_quantize_symmetric(gpu_ctx.handle, ctypes.c_void_p(xd.data_ptr()), m, k, mri.PER_TENSOR,
                                        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(s.data_ptr()))
        assert rc == 0, mri._lib.last_error()
        gpu_ctx.synchronize()
        want_q, want_s = oracle.quantize_symmetric(x)
        assert np.float32(s.item()) == want_s, rep
        assert np.array_equal(q.cpu().numpy().reshape(-1), want_q), rep
    gpu_ctx.check_device_status()


def test_one_launch_quantizer_feeds_gemm_exact(mri, oracle, gpu_ctx):
    """Consecutive prefill products on one stream (quantizer -> GEMM ->
    quantizer -> GEMM under programmatic dependent launch): each output
    bit-equal to the oracle."""
    rng = np.random.default_rng(90)
    m, n, k = 300, 1024, 4096
    wq, ws = weights(rng, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    import torch
    xs = [rng.normal(0, 1 + i, size=(m, k)).astype(np.float32) for i in range(3)]
    outs = [mri.matmul_int8_from_f32(torch.from_numpy(x).cuda(), qm) for x in xs]
    for x, o in zip(xs, outs):
        want, _, _, _ = oracle_from_f32(oracle, x, wq, ws, n, k)
        assert np.array_equal(bits(o.cpu().numpy()), bits(want))


# ── Q4_0 at one row: integer block dots, f32 for non-finite rows ─────────────

@pytest.mark.parametrize("limb", [1, 0])
@pytest.mark.parametrize("n,k", [(11008, 4096), (300, 1024), (7, 32), (2049, 8192), (64, 28672)])
def test_q4_0_one_row(mri, oracle, ctx_option, n, k, limb):
    """matmul_q4_0_dequant (q4_0.rs:94-181) at M = 1, on the integer kernel
    (OPT_Q4_LIMB = 1, K % 1024 == 0: 21-bit activation digits per block, exact
    dp4a block dots) and on the f32 streaming kernel (OPT_Q4_LIMB = 0, and
    K = 32 either way); within the Q4_0 bar of the reference's f32 sum,
    including rows whose activations span a wide range (a few large values,
    many tiny ones; blocks from 1e-30 to 1e30 and a block of subnormals)."""
    from test_gpu_parity import q4_close
    ctx_option(mri.OPT_Q4_LIMB, limb)
    rng = np.random.default_rng(n + k)
    wf = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    wb = oracle.quantize_q4_0_matrix(wf, n, k)
    wdeq = oracle.dequantize_q4_0(wb).reshape(n, k)
    # Blocks of 32 whose magnitudes run from 1e-30 to 1e30 (each block's own
    # power-of-two scale), and one block of subnormals.
    nb = k // 32
    spread = (rng.normal(0, 1, size=(nb, 32)) * 10.0 ** np.linspace(-30, 30, nb)[:, None]).astype(np.float32)
    spread[0] = rng.normal(0, 1e-39, size=32).astype(np.float32)
    for x in (rng.normal(0, 1, size=(1, k)).astype(np.float32),
              (rng.normal(0, 1e-3, size=(1, k)) * (rng.random((1, k)) < 0.99) +
               rng.normal(0, 50, size=(1, k)) * (rng.random((1, k)) >= 0.99)).astype(np.float32),
              spread.reshape(1, k),
              np.zeros((1, k), np.float32)):
        got = mri.matmul_q4_0_dequant(x, wb, n, k)
        want = oracle.matmul_q4_0_dequant(x, 1, k, wb, n, k)
        ok, worst = q4_close(got, want, x, wdeq)
        assert ok, worst


def test_q4_0_one_row_non_finite_takes_f32_path(mri, oracle):
    """An inf or a NaN in the activation row: the integer kernel switches to
    the f32 loop, so the outputs are non-finite exactly where the
    reference's are (q4_0.rs:94-181)."""
    rng = np.random.default_rng(77)
    n, k = 1000, 4096
    wb = oracle.quantize_q4_0_matrix(rng.normal(0, 0.02, size=(n, k)).astype(np.float32), n, k)
    for special in (np.inf, -np.inf, np.nan):
        x = rng.normal(0, 1, size=(1, k)).astype(np.float32)
        x[0, 123] = special
        got = mri.matmul_q4_0_dequant(x, wb, n, k)
        want = oracle.matmul_q4_0_dequant(x, 1, k, wb, n, k)
        assert np.array_equal(np.isnan(got), np.isnan(want)), special
        assert np.array_equal(np.isposinf(got), np.isposinf(want)), special
        assert np.array_equal(np.isneginf(got), np.isneginf(want)), special
