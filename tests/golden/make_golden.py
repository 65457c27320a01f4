"""Writes tests/golden/reference_known_answers.json.

The reference (mini-rust-inference, Rust) cannot be built or run in this
environment, so its parity anchor is its own unit tests: every case below
transcribes one reference test — its closed-form inputs, computed here in
IEEE float32 exactly as the Rust expression does, and the assertion it makes —
with the reference file:line it comes from.  The JSON is consumed by
tests/test_oracle_golden.py (CPU oracle) and tests/test_gpu_parity.py
(GPU C-ABI), so both are pinned to the same reference assertions.

Run:  python tests/golden/make_golden.py
"""
import json
import os

import numpy as np

F32 = np.float32


def affine(n, mul, add):
    """`(i as f32) * mul + add` for i in 0..n, each op rounded to f32."""
    i = np.arange(n, dtype=np.int64).astype(F32)
    return (i * F32(mul) + F32(add)).astype(F32)


def wrap_i8(v):
    return ((int(v) + 128) % 256) - 128


def floats(a):
    return [float(F32(v)) for v in np.asarray(a, dtype=F32).ravel()]


CASES = []


def case(**kw):
    CASES.append(kw)


# ── quant/int8/symmetric.rs ─────────────────────────────────────────────────
case(id="sym_doctest", src="src/quant/int8/symmetric.rs:35-39", op="quantize_symmetric",
     x=[0.0, 0.5, -1.0, 1.0],
     checks=[["scale_eq", float(F32(1.0) / F32(127.0))], ["q_at", 2, -127], ["q_at", 3, 127]])
case(id="sym_scale_max_abs", src="src/quant/int8/symmetric.rs:172-180", op="quantize_symmetric",
     x=floats([0.0, 2.54, -1.27, 1.0]),
     checks=[["scale_approx", float(F32(2.54) / F32(127.0)), 1e-6]])
case(id="sym_all_zero", src="src/quant/int8/symmetric.rs:183-188", op="quantize_symmetric",
     x=[0.0] * 16, checks=[["scale_eq", 1.0], ["q_all", 0]])
case(id="sym_negative_max", src="src/quant/int8/symmetric.rs:191-197", op="quantize_symmetric",
     x=floats([-3.81, 1.0, -0.5]),
     checks=[["scale_approx", float(F32(3.81) / F32(127.0)), 1e-5]])
case(id="sym_max_to_127", src="src/quant/int8/symmetric.rs:202-207", op="quantize_symmetric",
     x=[1.0, -1.0, 0.5], checks=[["q_at", 0, 127], ["q_at", 1, -127]])
case(id="sym_zero_to_zero", src="src/quant/int8/symmetric.rs:210-214", op="quantize_symmetric",
     x=[0.0, 1.0, -1.0], checks=[["q_at", 0, 0]])
case(id="sym_round_half_away", src="src/quant/int8/symmetric.rs:217-231", op="quantize_symmetric",
     x=[0.5, 1.0], checks=[["q_at", 1, 127], ["q_at", 0, 64]])
case(id="sym_clamp_boundary", src="src/quant/int8/symmetric.rs:234-242", op="quantize_symmetric",
     x=[100.0], checks=[["q_at", 0, 127]])
case(id="sym_roundtrip", src="src/quant/int8/symmetric.rs:247-263", op="quantize_symmetric",
     x=floats(np.arange(-64, 65).astype(F32) * F32(0.05)), checks=[["roundtrip_half_lsb", 1e-6]])
case(id="sym_into_equal", src="src/quant/int8/symmetric.rs:287-294", op="quantize_symmetric",
     x=floats(affine(64, 0.03, -1.0)), checks=[["into_equal"]])

# ── quant/int8/per_channel.rs ───────────────────────────────────────────────
case(id="pc_doctest", src="src/quant/int8/per_channel.rs:87-95", op="quantize_per_channel",
     w=floats([1.0, -2.0, 3.0, 0.1, 0.2, 0.3]), n_out=2, k_in=3,
     checks=[["scale_approx", 0, float(F32(3.0) / F32(127.0)), 1e-6],
             ["scale_approx", 1, float(F32(0.3) / F32(127.0)), 1e-6]])
case(id="pc_scale_per_row", src="src/quant/int8/per_channel.rs:244-252", op="quantize_per_channel",
     w=floats([1.0, -2.0, 3.0, 0.5, 0.0, 0.25]), n_out=2, k_in=3,
     checks=[["scale_approx", 0, float(F32(3.0) / F32(127.0)), 1e-5],
             ["scale_approx", 1, float(F32(0.5) / F32(127.0)), 1e-5]])
case(id="pc_zero_rows", src="src/quant/int8/per_channel.rs:255-261", op="quantize_per_channel",
     w=[0.0] * 6, n_out=2, k_in=3, checks=[["scale_eq", 0, 1.0], ["scale_eq", 1, 1.0], ["data_all", 0]])
case(id="pc_max_to_127", src="src/quant/int8/per_channel.rs:264-270", op="quantize_per_channel",
     w=[-5.0, 1.0, 2.5, 5.0], n_out=1, k_in=4, checks=[["data_at", 0, -127], ["data_at", 3, 127]])
case(id="pc_rows_independent", src="src/quant/int8/per_channel.rs:275-289", op="quantize_per_channel",
     w=[0.0, 0.0, 127.0, 0.0, 0.0, 1.0], n_out=2, k_in=3,
     checks=[["data_at", 2, 127], ["data_at", 5, 127],
             ["scale_approx", 0, 1.0, 1e-5], ["scale_approx", 1, float(F32(1.0) / F32(127.0)), 1e-5]])
case(id="pc_roundtrip", src="src/quant/int8/per_channel.rs:294-312", op="quantize_per_channel",
     w=floats(affine(128, 0.03, -2.0)), n_out=4, k_in=32, checks=[["roundtrip_half_lsb", 1e-6]])

# ── INT8 dot products: int8_avx2.rs / int8_neon.rs ─────────────────────────
case(id="dot_empty", src="src/ops/matmul/int8_avx2.rs:219-222", op="dot_i8", a=[], b=[], expect=0)
case(id="dot_tail_only", src="src/ops/matmul/int8_avx2.rs:225-230", op="dot_i8",
     a=[1, 2, 3], b=[4, 5, 6], expect=32)
case(id="dot_32_vs_scalar", src="src/ops/matmul/int8_avx2.rs:233-242", op="dot_i8",
     a=[wrap_i8(i - 16) for i in range(32)], b=[wrap_i8(wrap_i8(i * 2) - 30) for i in range(32)],
     expect="scalar")
case(id="dot_33_vs_scalar", src="src/ops/matmul/int8_avx2.rs:245-250", op="dot_i8",
     a=[wrap_i8(wrap_i8(i * 3) - 50) for i in range(33)],
     b=[wrap_i8(wrap_i8(i * 5) - 80) for i in range(33)], expect="scalar")
case(id="dot_all_positive", src="src/ops/matmul/int8_avx2.rs:253-258", op="dot_i8",
     a=[127] * 64, b=[1] * 64, expect=8128)
case(id="dot_mixed_signs", src="src/ops/matmul/int8_avx2.rs:261-268", op="dot_i8",
     a=[1 if i % 2 == 0 else -1 for i in range(64)], b=[2] * 64, expect=0)
case(id="dot_all_negative", src="src/ops/matmul/int8_avx2.rs:271-276", op="dot_i8",
     a=[-3] * 32, b=[-5] * 32, expect=480)
case(id="dot_large_k", src="src/ops/matmul/int8_avx2.rs:279-285", op="dot_i8",
     a=[127] * 4096, b=[1] * 4096, expect=127 * 4096)
case(id="dot_k128_vs_scalar", src="src/ops/matmul/int8_avx2.rs:288-297", op="dot_i8",
     a=[wrap_i8(wrap_i8(i * 7 + 3) - 64) for i in range(128)],
     b=[wrap_i8(wrap_i8(i * 11 + 1) - 64) for i in range(128)], expect="scalar")
case(id="dot_neon_tail5", src="src/ops/matmul/int8_neon.rs:208-214", op="dot_i8",
     a=[1, 2, 3, 4, 5], b=[5, 4, 3, 2, 1], expect=35)
case(id="dot_neon_16", src="src/ops/matmul/int8_neon.rs:217-222", op="dot_i8",
     a=[i - 8 for i in range(16)], b=[i - 7 for i in range(16)], expect="scalar")
case(id="dot_neon_17", src="src/ops/matmul/int8_neon.rs:225-230", op="dot_i8",
     a=[wrap_i8(wrap_i8(i * 3) - 25) for i in range(17)],
     b=[wrap_i8(wrap_i8(i * 5) - 40) for i in range(17)], expect="scalar")
case(id="dot_neon_all_negative", src="src/ops/matmul/int8_neon.rs:249-255", op="dot_i8",
     a=[-4] * 16, b=[-7] * 16, expect=448)

# ── ops/matmul/int8.rs (+ avx2 / parallel equivalence) ─────────────────────
case(id="i8_shape", src="src/ops/matmul/int8.rs:171-178", op="matmul_int8_from_f32",
     x=[0.5] * 96, m=3, k=32, w=floats(affine(64, 0.01, 0.0)), n_out=2, k_in=32,
     checks=[["shape", [3, 2]]])
case(id="i8_zero_input", src="src/ops/matmul/int8.rs:181-189", op="matmul_int8_from_f32",
     x=[0.0] * 64, m=2, k=32, w=floats(affine(128, 0.1, -6.0)), n_out=4, k_in=32,
     checks=[["all_abs_lt", 1e-6]])
case(id="i8_zero_weights", src="src/ops/matmul/int8.rs:192-201", op="matmul_int8_from_f32",
     x=floats(affine(96, 0.1, -5.0)), m=3, k=32, w=[0.0] * 64, n_out=2, k_in=32,
     checks=[["all_abs_lt", 1e-4]])
case(id="i8_vs_naive_small", src="src/ops/matmul/int8.rs:206-222", op="matmul_int8_from_f32",
     x=floats(affine(64, 0.05, -1.6)), m=2, k=32, w=floats(affine(128, 0.03, -2.0)), n_out=4, k_in=32,
     checks=[["vs_naive_rel", 0.02]])
case(id="i8_vs_naive_larger", src="src/ops/matmul/int8.rs:225-237", op="matmul_int8_from_f32",
     x=floats(affine(512, 0.02, -5.0)), m=4, k=128, w=floats(affine(1024, 0.01, -5.0)), n_out=8, k_in=128,
     checks=[["vs_naive_rel", 0.02]])
case(id="i8_single_dot", src="src/ops/matmul/int8.rs:240-252", op="matmul_int8_from_f32",
     x=[0.5] * 32, m=1, k=32, w=[1.0] * 32, n_out=1, k_in=32,
     checks=[["shape", [1, 1]], ["at", 0, 16.0, 0.5]])
case(id="i8_direct_eq_wrapper", src="src/ops/matmul/int8.rs:256-270", op="matmul_int8_from_f32",
     x=floats(affine(64, 0.06, -2.0)), m=2, k=32, w=floats(affine(96, 0.04, -2.0)), n_out=3, k_in=32,
     checks=[["direct_bit_equal"]])
case(id="i8_k_mismatch", src="src/ops/matmul/int8.rs:305-320", op="matmul_int8_from_f32",
     x=[1.0] * 32, m=1, k=32, w=[0.0] * 64, n_out=1, k_in=64, checks=[["error", "ShapeMismatch"]])
case(id="i8_k_match_ok", src="src/ops/matmul/int8.rs:305-311", op="matmul_int8_from_f32",
     x=[1.0] * 64, m=2, k=32, w=[0.0] * 64, n_out=2, k_in=32, checks=[["shape", [2, 2]]])
case(id="i8_bad_act_len", src="src/ops/matmul/int8.rs:323-331", op="matmul_int8",
     act_q=[0] * 10, act_scale=1.0, m=1, w=[0.0] * 64, n_out=2, k_in=32,
     checks=[["error", "InvalidShape"]])
case(id="i8_no_overflow_k4096", src="src/ops/matmul/int8.rs:335-353", op="matmul_int8_from_f32",
     x=[127.0] * 4096, m=1, k=4096, w=[127.0] * 4096, n_out=1, k_in=4096,
     checks=[["at_rel", 0, 127.0 * 127.0 * 4096.0, 0.02]])
case(id="avx2_vs_scalar_small", src="src/ops/matmul/int8_avx2.rs:323-336", op="matmul_int8_variants",
     x=floats(affine(64, 0.05, -1.6)), m=2, k=32, w=floats(affine(128, 0.03, -2.0)), n_out=4, k_in=32,
     checks=[["variants_rel", 1e-6]])
case(id="avx2_vs_scalar_k128", src="src/ops/matmul/int8_avx2.rs:339-353", op="matmul_int8_variants",
     x=floats(affine(512, 0.02, -5.0)), m=4, k=128, w=floats(affine(1024, 0.01, -5.0)), n_out=8, k_in=128,
     checks=[["variants_rel", 1e-6]])
case(id="par_small", src="src/ops/matmul/parallel.rs:380-393", op="matmul_int8_variants",
     x=floats(affine(256, 0.05, -1.6)), m=4, k=64, w=floats(affine(256, 0.03, -2.0)), n_out=4, k_in=64,
     checks=[["variants_rel", 1e-6]])
case(id="par_larger_k", src="src/ops/matmul/parallel.rs:395-408", op="matmul_int8_variants",
     x=floats(affine(16 * 256, 0.02, -5.0)), m=16, k=256, w=floats(affine(8 * 256, 0.01, -5.0)),
     n_out=8, k_in=256, checks=[["variants_rel", 1e-6]])
case(id="par_single_row", src="src/ops/matmul/parallel.rs:410-423", op="matmul_int8_variants",
     x=floats(affine(128, 0.06, -2.0)), m=1, k=128, w=floats(affine(6 * 128, 0.04, -2.0)),
     n_out=6, k_in=128, checks=[["variants_rel", 1e-6]])
_contam = np.zeros(8 * 64, dtype=F32)
_contam[3 * 64:4 * 64] = np.arange(64).astype(F32) * F32(0.1) + F32(0.5)
case(id="par_no_cross_row", src="src/ops/matmul/parallel.rs:439-458", op="matmul_int8_variants",
     x=floats(_contam), m=8, k=64, w=floats((np.arange(3 * 64) % 7).astype(F32) * F32(0.1)),
     n_out=3, k_in=64, checks=[["variants_rel", 1e-6], ["rows_zero_except", 3]])

# ── ops/matmul/q8_direct.rs ─────────────────────────────────────────────────
for cid, src, n_len, n_out, k_in, ok in [
        ("q8_raw_ok", "src/ops/matmul/q8_direct.rs:315-319", 68, 2, 32, True),
        ("q8_raw_k31", "src/ops/matmul/q8_direct.rs:322-326", 34, 1, 31, False),
        ("q8_raw_len33", "src/ops/matmul/q8_direct.rs:328-332", 33, 1, 32, False),
        ("q8_raw_n0", "src/ops/matmul/q8_direct.rs:334-338", 0, 0, 32, True)]:
    case(id=cid, src=src, op="q8_0_from_raw", data_len=n_len, n_out=n_out, k_in=k_in, ok=ok)
case(id="q8_shape", src="src/ops/matmul/q8_direct.rs:356-364", op="matmul_q8_0_direct",
     x=[0.5] * 96, m=3, k=32, w=floats(affine(128, 0.01, 0.0)), n_out=4, k_in=32,
     checks=[["shape", [3, 4]]])
case(id="q8_zero_input", src="src/ops/matmul/q8_direct.rs:366-376", op="matmul_q8_0_direct",
     x=[0.0] * 64, m=2, k=32, w=floats(affine(128, 0.1, -6.0)), n_out=4, k_in=32,
     checks=[["all_abs_lt", 1e-5]])
case(id="q8_zero_weights", src="src/ops/matmul/q8_direct.rs:378-389", op="matmul_q8_0_direct",
     x=floats(affine(64, 0.1, -3.0)), m=2, k=32, w=[0.0] * 64, n_out=2, k_in=32,
     checks=[["all_abs_lt", 1e-4]])
case(id="q8_vs_dequant_small", src="src/ops/matmul/q8_direct.rs:392-412", op="matmul_q8_0_direct",
     x=floats(affine(64, 0.05, -1.6)), m=2, k=32, w=floats(affine(128, 0.03, -2.0)), n_out=4, k_in=32,
     checks=[["vs_dequant_naive_rel", 0.03]])
case(id="q8_vs_dequant_multiblock", src="src/ops/matmul/q8_direct.rs:414-433", op="matmul_q8_0_direct",
     x=floats(affine(384, 0.02, -3.84)), m=3, k=128, w=floats(affine(768, 0.01, -3.84)), n_out=6, k_in=128,
     checks=[["vs_dequant_naive_rel", 0.03]])
case(id="q8_single_dot", src="src/ops/matmul/q8_direct.rs:435-447", op="matmul_q8_0_direct",
     x=[0.5] * 32, m=1, k=32, w=[1.0] * 32, n_out=1, k_in=32,
     checks=[["shape", [1, 1]], ["at", 0, 16.0, 1.0]])
case(id="q8_k_mismatch", src="src/ops/matmul/q8_direct.rs:480-495", op="matmul_q8_0_direct",
     x=[1.0] * 32, m=1, k=32, w=[0.0] * 128, n_out=2, k_in=64, checks=[["error", "ShapeMismatch"]])
case(id="q8_no_nan_inf", src="src/ops/matmul/q8_direct.rs:498-510", op="matmul_q8_0_direct",
     x=floats(affine(512, 0.02, -5.12)), m=16, k=32, w=floats(affine(1024, 0.01, -5.12)), n_out=32, k_in=32,
     checks=[["finite"]])

# ── ops/matmul/q4_0.rs ──────────────────────────────────────────────────────
case(id="q4_doctest", src="src/ops/matmul/q4_0.rs:25-40", op="matmul_q4_0",
     x=[1.0] * 64, m=2, k=32, w=floats(np.arange(32).astype(F32)), n_out=1, k_in=32,
     checks=[["shape", [2, 1]]])
case(id="q4_single_block", src="src/ops/matmul/q4_0.rs:215-237", op="matmul_q4_0",
     x=floats(affine(32, 0.05, 0.0)), m=1, k=32, w=floats(affine(32, 0.1, -1.5)), n_out=1, k_in=32,
     checks=[["vs_dequant_naive_abs", 1e-5]])
case(id="q4_multi_row", src="src/ops/matmul/q4_0.rs:240-268", op="matmul_q4_0",
     x=floats(affine(192, 0.01, 0.0)), m=3, k=64, w=floats(affine(256, 0.02, -0.5)), n_out=4, k_in=64,
     checks=[["shape", [3, 4]], ["vs_dequant_naive_abs", 1e-5]])
case(id="q4_zero_input", src="src/ops/matmul/q4_0.rs:270-281", op="matmul_q4_0",
     x=[0.0] * 64, m=2, k=32, w=[1.0] * 32, n_out=1, k_in=32, checks=[["all_abs_lt", 1e-5]])
case(id="q4_k_not_mult32", src="src/ops/matmul/q4_0.rs:318-326", op="matmul_q4_0",
     x=[1.0] * 33, m=1, k=33, w_len=18, n_out=1, k_in=33, checks=[["error", "InvalidShape"]])
case(id="q4_k_mismatch", src="src/ops/matmul/q4_0.rs:328-337", op="matmul_q4_0",
     x=[1.0] * 32, m=1, k=32, w_len=18, n_out=1, k_in=64, checks=[["error", "ShapeMismatch"]])
case(id="q4_wrong_len", src="src/ops/matmul/q4_0.rs:339-348", op="matmul_q4_0",
     x=[1.0] * 32, m=1, k=32, w_len=20, n_out=1, k_in=32, checks=[["error", "InvalidShape"]])
case(id="q4_output_shape", src="src/ops/matmul/q4_0.rs:350-358", op="matmul_q4_0",
     x=[0.0] * 640, m=5, k=128, w=[0.0] * 1024, n_out=8, k_in=128, checks=[["shape", [5, 8]]])
case(id="q4_larger", src="src/ops/matmul/q4_0.rs:360-390", op="matmul_q4_0",
     x=floats(affine(512, 0.005, 0.0)), m=4, k=128, w=floats(affine(1024, 0.01, -0.5)), n_out=8, k_in=128,
     checks=[["shape", [4, 8]], ["vs_dequant_naive_abs", 1e-5]])

# ── gguf/dequant.rs, gguf/quantization.rs codecs ───────────────────────────
def q8_block(h, quants):
    return [h & 0xFF, h >> 8] + [q & 0xFF for q in quants]


case(id="deq_q8_single", src="src/gguf/dequant.rs:762-784", op="dequantize_q8_0",
     data=q8_block(0x3C00, list(range(32))), checks=[["values_approx", floats(np.arange(32)), 1e-2]])
case(id="deq_q8_negative", src="src/gguf/dequant.rs:787-807", op="dequantize_q8_0",
     data=q8_block(0x3800, list(range(-16, 16))),
     checks=[["value_approx", 0, -8.0, 1e-2], ["value_approx", 16, 0.0, 1e-2], ["value_approx", 31, 7.5, 1e-2]])
case(id="deq_q8_two_blocks", src="src/gguf/dequant.rs:810-834", op="dequantize_q8_0",
     data=q8_block(0x3C00, [0] * 32) + q8_block(0x4000, [1] * 32),
     checks=[["values_approx", [0.0] * 32 + [2.0] * 32, 1e-2]])
case(id="deq_q8_bad_len", src="src/gguf/dequant.rs:837-844", op="dequantize_q8_0",
     data=[0] * 33, checks=[["error", "AlignmentError"]])
case(id="create_q8_roundtrip", src="src/gguf/dequant.rs:944-960", op="create_q8_0_block",
     values=floats(np.arange(32)), checks=[["roundtrip_abs", 0.5]])
case(id="create_q8_zeros", src="src/gguf/dequant.rs:963-971", op="create_q8_0_block",
     values=[0.0] * 32, checks=[["roundtrip_abs", 0.0]])
case(id="create_q8_negative", src="src/gguf/dequant.rs:974-984", op="create_q8_0_block",
     values=floats(np.arange(-16, 16)), checks=[["roundtrip_abs", 0.5]])
case(id="deq_q4_single", src="src/gguf/dequant.rs:1033-1061", op="dequantize_q4_0",
     data=[0x00, 0x3C] + [0x98] * 16, checks=[["values_approx", [0.0, 1.0] * 16, 0.1]])
case(id="deq_q4_doctest", src="src/gguf/dequant.rs:455-470", op="dequantize_q4_0",
     data=[0x00, 0x3C, 0x98] + [0] * 15,
     checks=[["value_approx", 0, 0.0, 0.1], ["value_approx", 1, 1.0, 0.1]])
case(id="deq_q4_negative", src="src/gguf/dequant.rs:1064-1086", op="dequantize_q4_0",
     data=[0x00, 0x40] + [0xF0] * 16,
     checks=[["value_approx", 0, -16.0, 0.1], ["value_approx", 1, 14.0, 0.1]])
case(id="deq_q4_bad_len", src="src/gguf/dequant.rs:1125-1132", op="dequantize_q4_0",
     data=[0] * 19, checks=[["error", "AlignmentError"]])
case(id="create_q4_roundtrip", src="src/gguf/dequant.rs:1246-1263", op="create_q4_0_block",
     values=floats(np.arange(-8, 24)), checks=[["roundtrip_abs", 3.0]])
case(id="create_q4_zeros", src="src/gguf/dequant.rs:1266-1274", op="create_q4_0_block",
     values=[0.0] * 32, checks=[["roundtrip_abs", 0.1], ["bytes_after_scale", 0x88]])
case(id="create_q4_small", src="src/gguf/dequant.rs:1277-1288", op="create_q4_0_block",
     values=floats((np.arange(32).astype(F32) - F32(16.0)) * F32(0.5)), checks=[["roundtrip_abs", 2.0]])
case(id="f16_roundtrip", src="src/gguf/quantization.rs:516-526", op="f16",
     values=[0.0, 1.0, -1.0, 0.5, 2.0, 100.0, -0.125, 65504.0])
case(id="f16_specials", src="src/gguf/quantization.rs:529-545", op="f16_specials",
     expect=[[0x0000, "0.0"], [0x8000, "-0.0"], [0x3C00, "1.0"], [0x7C00, "inf"], [0xFC00, "-inf"],
             [0x7C01, "nan"]])


def main():
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_known_answers.json")
    with open(out, "w") as f:
        json.dump({"generated_by": "tests/golden/make_golden.py",
                   "reference": "tamirkifle/mini-rust-inference (unit tests, transcribed)",
                   "cases": CASES}, f, indent=None, separators=(",", ":"))
        f.write("\n")
    print(f"wrote {len(CASES)} cases to {out}")


if __name__ == "__main__":
    main()
