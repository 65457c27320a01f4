"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bars (north_star): INT32 accumulators bit-exact; INT8 f32 outputs bit-exact
(the reference epilogue is reproduced exactly, which is tighter than the
1e-5 relative budget); Q8_0 bit-exact (block terms added in block order);
Q4_0 within 1e-3 relative of the reference's sequential f32 sum, with an
absolute floor of 1e-5 * sum_k |x_k * w_k| for outputs that cancel to ~0.
"""
import numpy as np
import pytest

from golden_checks import check_case, load_cases

pytestmark = pytest.mark.gpu

Q4_REL = 1e-3
Q4_FLOOR = 1e-5


class GpuImpl:
    """golden_checks interface over the product package (GPU)."""

    def __init__(self, mri, oracle):
        self.mri, self.o = mri, oracle

    def quantize_symmetric(self, x):
        return self.mri.quantize_symmetric(x)

    def quantize_per_channel(self, w, n, k):
        qm = self.mri.quantize_per_channel(w, n, k)
        return qm.data, qm.scales

    def dot_i8(self, a, b):
        k = a.size
        qm = self.mri.QuantizedMatrix(b, np.ones(1, np.float32), 1, k)
        acc = np.zeros((1, 1), dtype=np.int32)
        self.mri.matmul_int8(a, 1.0, qm, 1, acc_out=acc)
        return int(acc[0, 0])

    def matmul_int8_from_f32(self, x, m, k, wq, ws, n, k_in):
        qm = self.mri.QuantizedMatrix(wq, ws, n, k_in)
        return self.mri.matmul_int8_from_f32(np.asarray(x, np.float32).reshape(m, k), qm)

    def matmul_int8(self, aq, s, wq, ws, n, k_in, m):
        qm = self.mri.QuantizedMatrix(wq, ws, n, k_in)
        return self.mri.matmul_int8(aq, s, qm, m)

    def int8_variants(self):
        def wrap(fn):
            return lambda aq, s, wq, ws, n, k_in, m: fn(aq, s, self.mri.QuantizedMatrix(wq, ws, n, k_in), m)
        return [wrap(self.mri.matmul_int8_avx2), wrap(self.mri.matmul_int8_parallel)]

    def q8_0_from_raw_ok(self, n_len, n, k):
        try:
            self.mri.Q8_0WeightMatrix.from_raw_bytes(np.zeros(n_len, np.uint8), n, k)
            return True
        except self.mri.InvalidShape:
            return False

    def matmul_q8_0_direct(self, x, m, k, wb, n, k_in):
        w = self.mri.Q8_0WeightMatrix.from_raw_bytes(wb, n, k_in)
        return self.mri.matmul_q8_0_direct(np.asarray(x, np.float32).reshape(m, k), w)

    def matmul_q4_0(self, x, m, k, wb, n, k_in):
        return self.mri.matmul_q4_0_dequant(np.asarray(x, np.float32).reshape(m, k), wb, n, k_in)

    def q4_close(self, got, want, x, wdeq):
        return q4_close(got, want, x, wdeq)[0]

    def dequantize_q8_0(self, d):
        if np.asarray(d).size % 34:
            raise type("AlignmentError", (Exception,), {"kind": "AlignmentError"})()
        return self.mri.formats.dequantize_q8_0(d)

    def dequantize_q4_0(self, d):
        if np.asarray(d).size % 18:
            raise type("AlignmentError", (Exception,), {"kind": "AlignmentError"})()
        return self.mri.formats.dequantize_q4_0(d)

    def create_q8_0_block(self, v):
        return self.mri.formats.quantize_q8_0(v, 1, 32)

    def create_q4_0_block(self, v):
        return self.mri.formats.quantize_q4_0(v, 1, 32)

    def f16_to_f32(self, h):
        return self.mri.formats.f16_to_f32(np.array([h], np.uint16))[0]

    def f32_to_f16(self, f):
        return int(self.mri.formats.f32_to_f16_trunc(np.array([f], np.float32))[0])


CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_gpu_known_answer(case, mri, oracle, gpu_ctx):
    check_case(GpuImpl(mri, oracle), case, oracle)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def rand_case(rng, m, n, k, x_sigma=1.0):
    x = rng.normal(0, x_sigma, size=(m, k)).astype(np.float32)
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    return x, wq, ws


INT8_SHAPES = [(1, 11008, 4096), (1, 1, 16), (1, 7, 33), (2, 33, 32), (3, 100, 100), (4, 257, 4096),
               (5, 1000, 512), (6, 64, 48), (7, 129, 1024), (8, 511, 4096), (8, 3, 4099), (9, 40, 64),
               (17, 300, 256), (31, 130, 4096), (32, 16, 32), (64, 96, 128), (1, 5, 0)]


@pytest.mark.parametrize("m,n,k", INT8_SHAPES)
def test_int8_from_f32_bit_exact(m, n, k, mri, oracle, gpu_ctx):
    rng = np.random.default_rng(1000 + m * 7 + n + k)
    x, wq, ws = rand_case(rng, m, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    got = mri.matmul_int8_from_f32(x, qm)
    want = oracle.matmul_int8_from_f32(x, m, k, wq, ws, n, k)
    assert got.shape == (m, n)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("m,n,k", INT8_SHAPES)
def test_int8_prequantized_acc_bit_exact(m, n, k, mri, oracle, gpu_ctx):
    rng = np.random.default_rng(2000 + m + n * 3 + k)
    x, wq, ws = rand_case(rng, m, n, k)
    aq, s = oracle.quantize_symmetric(x)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    acc = np.zeros((m, n), dtype=np.int32)
    got = mri.matmul_int8(aq, s, qm, m, acc_out=acc)
    want, want_acc = oracle.matmul_int8(aq, s, wq, ws, n, k, m)
    assert np.array_equal(acc, want_acc)
    assert np.array_equal(bits(got), bits(want))


def test_int8_extreme_values(mri, oracle, gpu_ctx):
    """All +-127 (max |acc|) and -128 weights (reachable through the raw
    QuantizedMatrix fields) stay exact."""
    m, n, k = 4, 64, 4096
    aq = np.full(m * k, 127, np.int8)
    aq[k:2 * k] = -127
    wq = np.full(n * k, 127, np.int8)
    wq[: k] = -128
    ws = np.ones(n, np.float32)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    acc = np.zeros((m, n), np.int32)
    got = mri.matmul_int8(aq, np.float32(1.0), qm, m, acc_out=acc)
    want, want_acc = oracle.matmul_int8(aq, np.float32(1.0), wq, ws, n, k, m)
    assert np.array_equal(acc, want_acc) and np.array_equal(bits(got), bits(want))


def test_int8_device_tensors_match_host(mri, oracle, gpu_ctx):
    import torch
    rng = np.random.default_rng(5)
    m, n, k = 8, 2048, 4096
    x, wq, ws = rand_case(rng, m, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    xd = torch.from_numpy(x).cuda()
    got = mri.matmul_int8_from_f32(xd, qm)
    qm.ctx.synchronize()
    want = oracle.matmul_int8_from_f32(x, m, k, wq, ws, n, k)
    assert np.array_equal(bits(got.cpu().numpy()), bits(want))


@pytest.mark.parametrize("m,k", [(1, 4096), (8, 4096), (3, 100), (16, 4096), (512, 4096)])
def test_int8_per_row_granularity(m, k, mri, oracle, gpu_ctx):
    rng = np.random.default_rng(77 + m)
    n = 300
    x, wq, ws = rand_case(rng, m, n, k)
    x[1 % m] *= 50.0
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    got = mri.matmul_int8_from_f32(x, qm, granularity=1)
    for r in range(m):
        aq, s = oracle.quantize_symmetric(x[r])
        want, _ = oracle.matmul_int8(aq, s, wq, ws, n, k, 1)
        assert np.array_equal(bits(got[r:r + 1]), bits(want)), r


# (1001, 4099): more than four grid strides of float4s in the per-tensor pass
# (its unrolled loop, the remainder loop and a 3-element scalar tail).
@pytest.mark.parametrize("m,k", [(1, 4096), (8, 4096), (512, 4096), (3, 7), (1, 1), (64, 8192),
                                 (1001, 4099)])
def test_quantizer_bit_exact(m, k, mri, oracle, gpu_ctx):
    rng = np.random.default_rng(m * 31 + k)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    x.reshape(-1)[0] = 0.5 * np.abs(x).max()  # exercise exact half-way candidates
    q, s = mri.quantize_symmetric(x)
    q2, s2 = oracle.quantize_symmetric(x)
    assert np.float32(s) == s2 and np.array_equal(q, q2)
    qr, sr = mri.quantize_symmetric_rows(x, m, k)
    qr2, sr2 = oracle.quantize_symmetric_rows(x, m, k)
    assert np.array_equal(bits(sr), bits(sr2)) and np.array_equal(qr, qr2)


def test_quantizer_specials(mri, oracle, gpu_ctx):
    x = np.array([0.0, -0.0, np.nan, 1.0, -2.0, np.inf, 3.0, -np.inf], np.float32)
    for vals in (x[:2], x[:5], x, np.zeros(16, np.float32), np.array([np.nan, 1.0], np.float32)):
        q, s = mri.quantize_symmetric(vals)
        q2, s2 = oracle.quantize_symmetric(vals)
        assert np.array_equal(q, q2)
        assert (np.isnan(s) and np.isnan(s2)) or np.float32(s) == s2


def test_quantize_per_channel_matches_oracle(mri, oracle, gpu_ctx):
    rng = np.random.default_rng(9)
    n, k = 300, 1000
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    w[3] = 0
    qm = mri.quantize_per_channel(w, n, k)
    d2, s2 = oracle.quantize_per_channel(w, n, k)
    assert np.array_equal(qm.data, d2) and np.array_equal(bits(qm.scales), bits(s2))


# (1, 4096, 11008): nb = 344, a thread's units cross rows; (1, 300, 8192) and
# (3, 200, 11008): more terms than the registers hold (written straight into
# the term buffer), the latter on the streaming kernel at 3 rows (nb > 256).
Q8_SHAPES = [(1, 11008, 4096), (8, 11008, 4096), (1, 1, 32), (2, 33, 64), (3, 100, 96), (5, 77, 1024),
             (8, 9, 4096), (9, 50, 256), (1, 64, 28672), (4, 20, 40960), (16, 128, 512),
             (1, 4096, 11008), (1, 300, 8192), (3, 200, 11008)]


@pytest.mark.parametrize("m,n,k", Q8_SHAPES)
def test_q8_0_bit_exact(m, n, k, mri, oracle, gpu_ctx):
    rng = np.random.default_rng(3000 + m + n + k)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wb = oracle.quantize_q8_0_matrix(w, n, k)
    W = mri.Q8_0WeightMatrix.from_raw_bytes(wb, n, k)
    got = mri.matmul_q8_0_direct(x, W)
    want = oracle.matmul_q8_0_direct(x, m, k, wb, n, k)
    assert np.array_equal(bits(got), bits(want))


# M = 2..8 with K % 256 == 0 take the MMA Q8_0 kernel (activations quantized
# per row first) while three stages fit (K <= 5120); (2, 1000, 8192),
# (4, 300, 6144), (5, 71, 96) and (8, 40, 4128) exercise the fallbacks.
Q8_PIN_SHAPES = [(2, 1000, 8192), (4, 300, 6144), (3, 517, 2048), (7, 2049, 3072), (3, 333, 5120),
                 (6, 333, 5120), (8, 3, 1024), (2, 148 * 8 + 1, 4096), (5, 71, 96), (8, 40, 4096 + 32)]


@pytest.mark.parametrize("m,n,k", Q8_PIN_SHAPES)
def test_q8_0_multirow_bit_exact(m, n, k, mri, oracle, gpu_ctx):
    rng = np.random.default_rng(3500 + m + n + k)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    x[0, :] = 0.0            # zero row: scale 1.0
    x[m - 1, 5] = 1.0e4      # one large element dominates its row's scale
    wb = oracle.quantize_q8_0_matrix(w, n, k)
    W = mri.Q8_0WeightMatrix.from_raw_bytes(wb, n, k)
    got = mri.matmul_q8_0_direct(x, W)
    want = oracle.matmul_q8_0_direct(x, m, k, wb, n, k)
    assert np.array_equal(bits(got), bits(want))


def q4_close(got, want, x, wdeq):
    floor = Q4_FLOOR * (np.abs(x) @ np.abs(wdeq).T)
    err = np.abs(got - want)
    return np.all(err <= np.maximum(Q4_REL * np.abs(want), floor)), float(np.max(err / np.maximum(np.abs(want), 1e-30)))


@pytest.mark.parametrize("m,n,k", Q8_SHAPES)
def test_q4_0_within_tolerance(m, n, k, mri, oracle, gpu_ctx):
    rng = np.random.default_rng(4000 + m + n + k)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wb = oracle.quantize_q4_0_matrix(w, n, k)
    got = mri.matmul_q4_0_dequant(x, wb, n, k)
    want = oracle.matmul_q4_0_dequant(x, m, k, wb, n, k)
    ok, worst = q4_close(got, want, x, oracle.dequantize_q4_0(wb).reshape(n, k))
    assert ok, worst


# M = 2..8 with K % 256 == 0 take the bf16-MMA Q4_0 kernel while the split
# activations and three stages fit; (4, 20, 40960) and (3, 50, 96) fall back.
Q4_MMA_SHAPES = [(3, 517, 2048), (7, 2049, 3072), (2, 148 * 8 + 1, 4096), (6, 333, 5120),
                 (8, 40, 256), (8, 11008, 4096), (4, 20, 40960), (3, 50, 96)]


@pytest.mark.parametrize("m,n,k", Q4_MMA_SHAPES)
def test_q4_0_multirow_within_tolerance(m, n, k, mri, oracle, gpu_ctx):
    rng = np.random.default_rng(4500 + m + n + k)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    x[0, :] = 0.0            # a zero row
    x[m - 1, 7] = 3.0e4      # one large element
    wb = oracle.quantize_q4_0_matrix(w, n, k)
    got = mri.matmul_q4_0_dequant(x, wb, n, k)
    want = oracle.matmul_q4_0_dequant(x, m, k, wb, n, k)
    ok, worst = q4_close(got, want, x, oracle.dequantize_q4_0(wb).reshape(n, k))
    assert ok, worst


def test_sharded_equals_unsharded(mri, oracle, gpu_ctx):
    """An N-column shard computes bit-identical columns (the per-(m, n)
    arithmetic does not depend on the other rows of W)."""
    rng = np.random.default_rng(11)
    m, n, k = 3, 1376 * 4 + 5, 4096
    x, wq, ws = rand_case(rng, m, n, k)
    full = mri.matmul_int8_from_f32(x, mri.QuantizedMatrix(wq, ws, n, k))
    parts = []
    P = 4
    for r in range(P):
        b, e = n * r // P, n * (r + 1) // P
        parts.append(mri.matmul_int8_from_f32(x, mri.QuantizedMatrix(wq, ws, n, k, rows=(b, e))))
    assert np.array_equal(bits(np.concatenate(parts, axis=1)), bits(full))


def test_prefill_shape_sampled_rows_exact(mri, oracle, gpu_ctx):
    """BASELINE prefill config [512,4096]x[4096,11008]: all INT32 accumulators
    of 12 sampled rows equal the oracle's; the per-tensor scale is global."""
    rng = np.random.default_rng(1)
    m, n, k = 512, 11008, 4096
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wf = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    wq, ws = oracle.quantize_per_channel(wf, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    aq, s = oracle.quantize_symmetric(x)
    acc = np.zeros((m, n), np.int32)
    got = mri.matmul_int8(aq, s, qm, m, acc_out=acc)
    rows = rng.choice(m, size=12, replace=False)
    sub = aq.reshape(m, k)[rows].reshape(-1)
    want, want_acc = oracle.matmul_int8(sub, s, wq, ws, n, k, len(rows))
    assert np.array_equal(acc[rows], want_acc)
    assert np.array_equal(bits(got[rows]), bits(want))


@pytest.mark.parametrize("bn", [128, 160, 192, 224, 256])
def test_gemm_tile_widths_exact(mri, oracle, ctx_option, bn):
    """Every tensor-core tile width (OPT_GEMM_BN) gives the oracle's INT32
    sums and f32 outputs on ragged M and N, with a residual-free epilogue."""
    ctx_option(mri.OPT_GEMM_BN, bn)
    rng = np.random.default_rng(100 + bn)
    m, n, k = 333, 1000, 4096 + 256
    aq = rng.integers(-127, 128, size=m * k, dtype=np.int8)
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    acc = np.zeros((m, n), np.int32)
    got = mri.matmul_int8(aq, np.float32(0.0123), qm, m, acc_out=acc)
    want, want_acc = oracle.matmul_int8(aq, np.float32(0.0123), wq, ws, n, k, m)
    assert np.array_equal(acc, want_acc)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("bn", [128, 160])
def test_gemm_two_ctas_per_sm_exact(mri, oracle, ctx_option, bn):
    """Between one and two rounds of tiles (here 196 or 244 tiles on 148 SMs)
    the GEMM runs one tile per CTA, two CTAs per SM: same INT32 sums and f32
    outputs as the oracle on ragged M and N."""
    ctx_option(mri.OPT_GEMM_BN, bn)
    rng = np.random.default_rng(200 + bn)
    m, n, k = 500, 7717, 1024 + 256
    aq = rng.integers(-127, 128, size=m * k, dtype=np.int8)
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    acc = np.zeros((m, n), np.int32)
    got = mri.matmul_int8(aq, np.float32(0.0123), qm, m, acc_out=acc)
    want, want_acc = oracle.matmul_int8(aq, np.float32(0.0123), wq, ws, n, k, m)
    assert np.array_equal(acc, want_acc)
    assert np.array_equal(bits(got), bits(want))


# The epilogue stages each warp's 32 x 32 output block in shared memory when the
# block lies inside M and N and no INT32 copy is requested (acc_out selects the
# direct per-row stores); the cases below leave acc_out out so that the staged
# stores are the ones checked, on full and ragged blocks.
@pytest.mark.parametrize("pair", [0, 2], ids=["one_cta", "cta_pair"])
@pytest.mark.parametrize("bn", [128, 160, 192, 224, 256])
def test_gemm_staged_epilogue_exact(mri, oracle, ctx_option, bn, pair):
    """Plain outputs (no INT32 copy): the staged stores of the one-CTA kernel
    (OPT_GEMM_PAIR = 0) and of the CTA-pair kernel (256-row tiles on
    tcgen05.mma.cta_group::2), every tile width."""
    ctx_option(mri.OPT_GEMM_BN, bn)
    ctx_option(mri.OPT_GEMM_PAIR, pair)
    rng = np.random.default_rng(300 + bn)
    m, n, k = 333, 1000, 4096 + 256
    aq = rng.integers(-127, 128, size=m * k, dtype=np.int8)
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    got = mri.matmul_int8(aq, np.float32(0.0123), qm, m)
    want, _ = oracle.matmul_int8(aq, np.float32(0.0123), wq, ws, n, k, m)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("bn", [128, 160])
def test_gemm_two_ctas_per_sm_staged_exact(mri, oracle, ctx_option, bn):
    """One tile per CTA, two CTAs per SM: the output block is staged in the
    (then idle) stage ring."""
    ctx_option(mri.OPT_GEMM_BN, bn)
    ctx_option(mri.OPT_GEMM_PAIR, 0)
    rng = np.random.default_rng(400 + bn)
    m, n, k = 500, 7717, 1024 + 256
    aq = rng.integers(-127, 128, size=m * k, dtype=np.int8)
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    got = mri.matmul_int8(aq, np.float32(0.0123), qm, m)
    want, _ = oracle.matmul_int8(aq, np.float32(0.0123), wq, ws, n, k, m)
    assert np.array_equal(bits(got), bits(want))


def test_prefill_shape_f32_exact(mri, oracle, gpu_ctx):
    """BASELINE prefill config through matmul_int8_from_f32 (per-tensor
    quantizer + tensor-core GEMM with the staged epilogue): 16 sampled rows
    bit-equal to the oracle's."""
    rng = np.random.default_rng(11)
    m, n, k = 512, 11008, 4096
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    got = mri.matmul_int8_from_f32(x, qm)
    aq, s = oracle.quantize_symmetric(x)
    rows = np.sort(np.concatenate([[0, 31, 32, 127, 128, 511], rng.choice(m, size=10, replace=False)]))
    want, _ = oracle.matmul_int8(aq.reshape(m, k)[rows].reshape(-1), s, wq, ws, n, k, len(rows))
    assert np.array_equal(bits(got[rows]), bits(want))


def _transposed_input(scale, offset, on_device):
    """The reference's non-contiguous input: the [2, 64] transpose of a
    row-major [64, 2] tensor holding i * scale + offset.  Returns the view, its
    contiguous copy (same residency) and the contiguous host values."""
    t = (np.arange(128, dtype=np.float32) * np.float32(scale) + np.float32(offset)).reshape(64, 2)
    host = np.ascontiguousarray(t.T)
    if on_device:
        import torch
        nc = torch.from_numpy(t).cuda().t()
        assert not nc.is_contiguous()
        return nc, nc.contiguous(), host
    nc = t.T
    assert not nc.flags["C_CONTIGUOUS"]
    return nc, np.ascontiguousarray(nc), host


def _to_host(a):
    return a.cpu().numpy() if hasattr(a, "cpu") else np.asarray(a)


@pytest.mark.parametrize("on_device", [False, True], ids=["host", "device"])
def test_non_contiguous_inputs_match_contiguous(mri, oracle, gpu_ctx, on_device):
    """int8.rs:274-288, q8_direct.rs:449-464, q4_0.rs:283-303: a transposed
    [2, 64] input gives bit for bit the outputs of its contiguous copy, and the
    oracle's (Q4_0 within the Q4_0 bar), for host arrays and CUDA tensors."""
    # INT8 (int8.rs:276-286)
    nc, c, xh = _transposed_input(0.05, -3.0, on_device)
    w = np.arange(192, dtype=np.float32) * np.float32(0.02) - np.float32(2.0)
    qw = mri.quantize_per_channel(w, 3, 64)
    got_nc = _to_host(mri.matmul_int8_from_f32(nc, qw))
    got_c = _to_host(mri.matmul_int8_from_f32(c, qw))
    assert np.array_equal(bits(got_nc), bits(got_c))
    want = oracle.matmul_int8_from_f32(xh, 2, 64, qw.data, qw.scales, 3, 64)
    assert np.array_equal(bits(got_nc), bits(want))
    # Q8_0 (q8_direct.rs:451-463)
    qw8 = mri.Q8_0WeightMatrix.from_f32_tensor(w.reshape(3, 64))
    got_nc = _to_host(mri.matmul_q8_0_direct(nc, qw8))
    got_c = _to_host(mri.matmul_q8_0_direct(c, qw8))
    assert np.array_equal(bits(got_nc), bits(got_c))
    want = oracle.matmul_q8_0_direct(xh, 2, 64, qw8.data, 3, 64)
    assert np.array_equal(bits(got_nc), bits(want))
    # Q4_0 (q4_0.rs:285-302)
    nc, c, xh = _transposed_input(0.01, 0.0, on_device)
    w4 = ((np.arange(3)[:, None] + np.arange(64)[None, :]).astype(np.float32) * np.float32(0.03)
          - np.float32(0.5))
    wb = oracle.quantize_q4_0_matrix(w4, 3, 64)
    got_nc = _to_host(mri.matmul_q4_0_dequant(nc, wb, 3, 64))
    got_c = _to_host(mri.matmul_q4_0_dequant(c, wb, 3, 64))
    assert got_nc.shape == (2, 3)
    assert np.array_equal(bits(got_nc), bits(got_c))
    want = oracle.matmul_q4_0_dequant(xh, 2, 64, wb, 3, 64)
    ok, worst = q4_close(got_nc, want, xh, oracle.dequantize_q4_0(wb).reshape(3, 64))
    assert ok, worst


def test_device_inputs_ordered_with_torch_stream(mri, oracle, gpu_ctx):
    """A context's stream is non-blocking.  An input that torch is still
    writing on its current stream when the call is made must be complete
    before the kernels read it, and torch must see the finished output, with
    no explicit synchronization in between."""
    import torch
    rng = np.random.default_rng(21)
    m, n, k = 4, 1024, 4096
    x, wq, ws = rand_case(rng, m, n, k)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    src = torch.from_numpy(x).cuda()
    xd = torch.zeros(m, k, device="cuda")
    torch.cuda.synchronize()
    torch.cuda._sleep(2_000_000)  # keep torch's stream busy (about a millisecond) ...
    xd.copy_(src)                 # ... so that the input is written late
    got = (mri.matmul_int8_from_f32(xd, qm) * 1.0).cpu().numpy()
    want = oracle.matmul_int8_from_f32(x, m, k, wq, ws, n, k)
    assert np.array_equal(bits(got), bits(want))


def test_device_status_clean(mri, gpu_ctx):
    """No bounded device-side wait gave up during the tests above."""
    gpu_ctx.check_device_status()


@pytest.mark.parametrize("m", [1, 3])
def test_host_calls_with_pinned_buffers(mri, oracle, gpu_ctx, m):
    """The host-buffer entry points write a pinned (page-locked, mapped)
    output through a copy kernel on its device mapping instead of a
    device-to-host copy: the results equal the reference's, and the same call
    on pageable memory, bit for bit, also after the caller rewrites the
    pinned input in place."""
    import ctypes
    import torch
    lib = mri._lib.load()
    rng = np.random.default_rng(77 + m)
    n, k = 1000, 4096
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wq, ws = rng.integers(-127, 128, size=n * k, dtype=np.int8), rng.uniform(0.001, 0.02, n).astype(np.float32)
    wf = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    qm = mri.QuantizedMatrix(wq, ws, n, k)
    q8 = mri.Q8_0WeightMatrix.from_raw_bytes(oracle.quantize_q8_0_matrix(wf, n, k), n, k)
    q4b = oracle.quantize_q4_0_matrix(wf, n, k)
    q4 = mri.Q4_0Matrix(q4b, n, k)
    x_pin = torch.empty(m, k).pin_memory()
    for x in (x, rng.normal(0, 3, size=(m, k)).astype(np.float32)):
        x_pin.copy_(torch.from_numpy(x))  # rewritten in place for the second round
        cases = [(lib.mri_host_matmul_int8_from_f32, qm, mri.matmul_int8_from_f32(x, qm)),
                 (lib.mri_host_matmul_q8_0_direct, q8, mri.matmul_q8_0_direct(x, q8)),
                 (lib.mri_host_matmul_q4_0_dequant, q4, mri.matmul_q4_0_dequant(x, q4b, n, k))]
        for fn, w, pageable in cases:
            out = torch.full((m, n), float("nan")).pin_memory()
            rc = fn(gpu_ctx.handle, ctypes.c_void_p(x_pin.data_ptr()), m, k, w.handle,
                    ctypes.c_void_p(out.data_ptr()))
            assert rc == 0, mri._lib.last_error()
            assert np.array_equal(bits(out.numpy()), bits(np.asarray(pageable, np.float32))), fn
        want = oracle.matmul_int8_from_f32(x, m, k, wq, ws, n, k)
        assert np.array_equal(bits(cases[0][2]), bits(want))
    # A pinned output that is not 16-byte aligned is copied instead.
    buf = torch.full((m * n + 1,), float("nan")).pin_memory()
    rc = lib.mri_host_matmul_int8_from_f32(gpu_ctx.handle, ctypes.c_void_p(x_pin.data_ptr()), m, k, qm.handle,
                                           ctypes.c_void_p(buf.data_ptr() + 4))
    assert rc == 0, mri._lib.last_error()
    assert np.array_equal(bits(buf[1:].numpy().reshape(m, n)), bits(np.asarray(cases[0][2], np.float32)))
