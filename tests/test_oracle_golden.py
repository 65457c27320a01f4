"""Pins the CPU oracle to the reference's own unit-test assertions."""
import numpy as np
import pytest

from golden_checks import check_case, load_cases


class OracleImpl:
    """Adapts oracle.py to the interface golden_checks expects."""

    def __init__(self, o):
        self.o = o

    def quantize_symmetric(self, x):
        return self.o.quantize_symmetric(x)

    def quantize_per_channel(self, w, n, k):
        return self.o.quantize_per_channel(w, n, k)

    def dot_i8(self, a, b):
        got = self.o.dot_i8_avx2(a, b)
        assert got == self.o.dot_i8_scalar(a, b)
        return got

    def matmul_int8_from_f32(self, x, m, k, wq, ws, n, k_in):
        return self.o.matmul_int8_from_f32(x, m, k, wq, ws, n, k_in)

    def matmul_int8(self, aq, s, wq, ws, n, k_in, m):
        return self.o.matmul_int8(aq, s, wq, ws, n, k_in, m)[0]

    def int8_variants(self):
        o = self.o
        return [o.matmul_int8_avx2,
                lambda *a: o.matmul_int8_parallel(*a, n_threads=4)]

    def q8_0_from_raw_ok(self, n_len, n, k):
        return self.o.q8_0_check_raw(n_len, n, k) == 0

    def matmul_q8_0_direct(self, x, m, k, wb, n, k_in):
        return self.o.matmul_q8_0_direct(x, m, k, wb, n, k_in)

    def matmul_q4_0(self, x, m, k, wb, n, k_in):
        return self.o.matmul_q4_0_dequant(x, m, k, wb, n, k_in)

    def dequantize_q8_0(self, d):
        return self.o.dequantize_q8_0(d)

    def dequantize_q4_0(self, d):
        return self.o.dequantize_q4_0(d)

    def create_q8_0_block(self, v):
        return self.o.create_q8_0_block(v)

    def create_q4_0_block(self, v):
        return self.o.create_q4_0_block(v)

    def f16_to_f32(self, h):
        return self.o.f16_to_f32(h)

    def f32_to_f16(self, f):
        return self.o.f32_to_f16(f)


CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_oracle_known_answer(case, oracle):
    check_case(OracleImpl(oracle), case, oracle)


def test_parallel_bit_identical_to_scalar(oracle):
    """parallel.rs:361 states bit-identity with the scalar kernel; check it on a
    random case with odd sizes (tail handling in the AVX2 dot)."""
    rng = np.random.default_rng(7)
    m, n, k = 5, 37, 4099
    aq = rng.integers(-127, 128, size=m * k, dtype=np.int8)
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    s = np.float32(0.0123)
    ref, _ = oracle.matmul_int8(aq, s, wq, ws, n, k, m)
    par = oracle.matmul_int8_parallel(aq, s, wq, ws, n, k, m, n_threads=3)
    assert np.array_equal(ref.view(np.uint32), par.view(np.uint32))


def test_neon_and_avx2_agree(oracle):
    """int8_neon.rs:318-332 on the reference's inputs.  Off aarch64 the NEON
    kernel's dot is the scalar one (int8_neon.rs:126-131); every dot is an
    exact INT32 sum, so the AVX2 outputs equal the scalar outputs bit for bit
    (the reference asks for a relative error below 1e-6)."""
    k, n, m = 128, 6, 4
    w = np.arange(n * k, dtype=np.float32) * np.float32(0.01) - np.float32(5.0)
    inp = np.arange(m * k, dtype=np.float32) * np.float32(0.02) - np.float32(5.0)
    wq, ws = oracle.quantize_per_channel(w, n, k)
    aq, s = oracle.quantize_symmetric(inp)
    scalar, _ = oracle.matmul_int8(aq, s, wq, ws, n, k, m)
    avx2 = oracle.matmul_int8_avx2(aq, s, wq, ws, n, k, m)
    assert np.array_equal(scalar.view(np.uint32), avx2.view(np.uint32))


def test_f16_exhaustive_against_numpy(oracle):
    """f16_to_f32 (quantization.rs:416-461) is exact for every non-NaN code."""
    for h in range(0, 1 << 16, 7):
        got = oracle.f16_to_f32(h)
        want = np.array([h], dtype=np.uint16).view(np.float16).astype(np.float32)[0]
        if np.isnan(want):
            assert np.isnan(got)
        else:
            assert got == want and np.signbit(got) == np.signbit(want), h


def test_f32_to_f16_truncates(oracle):
    """quantization.rs:464-498 truncates the mantissa (mant >> 13)."""
    assert oracle.f32_to_f16(1.0) == 0x3C00
    # 1 + 0.75 ulp(f16): round-to-nearest would give 0x3C01, truncation 0x3C00
    assert oracle.f32_to_f16(np.float32(1.0) + np.float32(2 ** -11) + np.float32(2 ** -12)) == 0x3C00
    assert oracle.f32_to_f16(70000.0) == 0x7C00
    assert oracle.f32_to_f16(1e-9) == 0x0000
