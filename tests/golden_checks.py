"""Evaluates the reference's transcribed known answers
(tests/golden/reference_known_answers.json) against an implementation.

An implementation is any object with the methods used below; tests pass the
CPU oracle (tests/test_oracle_golden.py) or the GPU C-ABI
(tests/test_gpu_parity.py).  Errors are exceptions with a `.kind` attribute
naming the reference's TensorError variant.
"""
import json
import math
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                      "reference_known_answers.json")


def load_cases(ops=None):
    with open(GOLDEN) as f:
        cases = json.load(f)["cases"]
    if ops is not None:
        cases = [c for c in cases if c["op"] in ops]
    return cases


def max_rel_err(a, b):
    """The reference tests' metric (e.g. src/ops/matmul/int8.rs:146-154)."""
    a = np.asarray(a, dtype=np.float32).ravel()
    b = np.asarray(b, dtype=np.float32).ravel()
    denom = np.maximum(np.maximum(np.abs(a), np.abs(b)), np.float32(1e-3))
    return float(np.max(np.abs(a - b) / denom)) if a.size else 0.0


def naive_matmul_t(x, w, m, k, n):
    """matmul_naive(input, w^T) (src/ops/matmul/naive.rs): sequential f32 sum over k."""
    x = np.asarray(x, dtype=np.float32).reshape(m, k)
    w = np.asarray(w, dtype=np.float32).reshape(n, k)
    out = np.zeros((m, n), dtype=np.float32)
    for i in range(m):
        for j in range(n):
            acc = np.float32(0.0)
            for t in range(k):
                acc = np.float32(acc + np.float32(x[i, t] * w[j, t]))
            out[i, j] = acc
    return out


def _expect_error(fn, kind):
    try:
        fn()
    except Exception as e:  # noqa: BLE001 - any implementation error type
        got = getattr(e, "kind", type(e).__name__)
        assert got == kind, f"expected {kind}, got {got}"
        return
    raise AssertionError(f"expected error {kind}, call succeeded")


def check_case(impl, c, oracle):
    op = c["op"]
    checks = c.get("checks", [])
    if op == "quantize_symmetric":
        q, s = impl.quantize_symmetric(np.array(c["x"], dtype=np.float32))
        q = np.asarray(q)
        for ch in checks:
            if ch[0] == "scale_eq":
                assert np.float32(s) == np.float32(ch[1]), (s, ch[1])
            elif ch[0] == "scale_approx":
                assert abs(float(s) - ch[1]) < ch[2], (s, ch[1])
            elif ch[0] == "q_at":
                assert int(q[ch[1]]) == ch[2], (q[ch[1]], ch[2])
            elif ch[0] == "q_all":
                assert np.all(q == ch[1])
            elif ch[0] == "roundtrip_half_lsb":
                rec = q.astype(np.float32) * np.float32(s)
                err = np.max(np.abs(np.array(c["x"], dtype=np.float32) - rec))
                assert err <= float(s) / 2 + ch[1], (err, s)
            elif ch[0] == "into_equal":
                q2, s2 = oracle.quantize_symmetric(np.array(c["x"], dtype=np.float32))
                assert np.array_equal(q, q2) and np.float32(s) == s2
            else:
                raise KeyError(ch[0])
    elif op == "quantize_per_channel":
        data, scales = impl.quantize_per_channel(np.array(c["w"], dtype=np.float32), c["n_out"], c["k_in"])
        data, scales = np.asarray(data).ravel(), np.asarray(scales)
        for ch in checks:
            if ch[0] == "scale_approx":
                assert abs(float(scales[ch[1]]) - ch[2]) < ch[3]
            elif ch[0] == "scale_eq":
                assert scales[ch[1]] == np.float32(ch[2])
            elif ch[0] == "data_at":
                assert int(data[ch[1]]) == ch[2]
            elif ch[0] == "data_all":
                assert np.all(data == ch[1])
            elif ch[0] == "roundtrip_half_lsb":
                w = np.array(c["w"], dtype=np.float32).reshape(c["n_out"], c["k_in"])
                rec = data.reshape(c["n_out"], c["k_in"]).astype(np.float32) * scales[:, None]
                for r in range(c["n_out"]):
                    assert np.max(np.abs(w[r] - rec[r])) <= scales[r] / 2 + ch[1]
            else:
                raise KeyError(ch[0])
    elif op == "dot_i8":
        got = impl.dot_i8(np.array(c["a"], dtype=np.int8), np.array(c["b"], dtype=np.int8))
        if c["expect"] == "scalar":
            exp = int(np.dot(np.array(c["a"], dtype=np.int64), np.array(c["b"], dtype=np.int64)))
        else:
            exp = c["expect"]
        assert got == exp, (got, exp)
    elif op in ("matmul_int8_from_f32", "matmul_int8_variants"):
        m, k, n, k_in = c["m"], c["k"], c["n_out"], c["k_in"]
        x = np.array(c["x"], dtype=np.float32)
        w = np.array(c["w"], dtype=np.float32)
        wq, ws = oracle.quantize_per_channel(w, n, k_in)
        errs = [ch for ch in checks if ch[0] == "error"]
        if errs:
            _expect_error(lambda: impl.matmul_int8_from_f32(x, m, k, wq, ws, n, k_in), errs[0][1])
            return
        out = np.asarray(impl.matmul_int8_from_f32(x, m, k, wq, ws, n, k_in))
        for ch in checks:
            if ch[0] == "shape":
                assert list(out.shape) == ch[1], (out.shape, ch[1])
            elif ch[0] == "all_abs_lt":
                assert np.all(np.abs(out) < ch[1])
            elif ch[0] == "vs_naive_rel":
                ref = naive_matmul_t(x, w, m, k, n)
                assert max_rel_err(out, ref) < ch[1]
            elif ch[0] == "at":
                assert abs(float(out.ravel()[ch[1]]) - ch[2]) < ch[3]
            elif ch[0] == "at_rel":
                assert abs(float(out.ravel()[ch[1]]) - ch[2]) / ch[2] < ch[3]
            elif ch[0] == "direct_bit_equal":
                aq, s = oracle.quantize_symmetric(x)
                direct = np.asarray(impl.matmul_int8(aq, s, wq, ws, n, k_in, m))
                assert np.array_equal(direct.view(np.uint32), out.view(np.uint32))
            elif ch[0] == "variants_rel":
                aq, s = oracle.quantize_symmetric(x)
                scalar, _ = oracle.matmul_int8(aq, s, wq, ws, n, k_in, m)
                assert max_rel_err(out, scalar) < ch[1]
                for variant in impl.int8_variants():
                    got = np.asarray(variant(aq, s, wq, ws, n, k_in, m))
                    assert max_rel_err(got, scalar) < ch[1]
            elif ch[0] == "rows_zero_except":
                for r in range(m):
                    if r != ch[1]:
                        assert np.all(out[r] == 0)
            else:
                raise KeyError(ch[0])
    elif op == "matmul_int8":
        n, k_in, m = c["n_out"], c["k_in"], c["m"]
        wq, ws = oracle.quantize_per_channel(np.array(c["w"], dtype=np.float32), n, k_in)
        aq = np.array(c["act_q"], dtype=np.int8)
        for ch in checks:
            assert ch[0] == "error"
            _expect_error(lambda: impl.matmul_int8(aq, c["act_scale"], wq, ws, n, k_in, m), ch[1])
    elif op == "q8_0_from_raw":
        ok = impl.q8_0_from_raw_ok(c["data_len"], c["n_out"], c["k_in"])
        assert ok == c["ok"], (ok, c["ok"])
    elif op == "matmul_q8_0_direct":
        m, k, n, k_in = c["m"], c["k"], c["n_out"], c["k_in"]
        x = np.array(c["x"], dtype=np.float32)
        w = np.array(c["w"], dtype=np.float32)
        wb = oracle.quantize_q8_0_matrix(w, n, k_in)
        errs = [ch for ch in checks if ch[0] == "error"]
        if errs:
            _expect_error(lambda: impl.matmul_q8_0_direct(x, m, k, wb, n, k_in), errs[0][1])
            return
        out = np.asarray(impl.matmul_q8_0_direct(x, m, k, wb, n, k_in))
        for ch in checks:
            if ch[0] == "shape":
                assert list(out.shape) == ch[1]
            elif ch[0] == "all_abs_lt":
                assert np.all(np.abs(out) < ch[1])
            elif ch[0] == "vs_dequant_naive_rel":
                ref = naive_matmul_t(x, oracle.dequantize_q8_0(wb), m, k, n)
                assert max_rel_err(out, ref) < ch[1]
            elif ch[0] == "at":
                assert abs(float(out.ravel()[ch[1]]) - ch[2]) < ch[3]
            elif ch[0] == "finite":
                assert np.all(np.isfinite(out))
            else:
                raise KeyError(ch[0])
    elif op == "matmul_q4_0":
        m, k, n, k_in = c["m"], c["k"], c["n_out"], c["k_in"]
        x = np.array(c["x"], dtype=np.float32)
        if "w" in c:
            wb = oracle.quantize_q4_0_matrix(np.array(c["w"], dtype=np.float32), n, k_in)
        else:
            wb = np.zeros(c["w_len"], dtype=np.uint8)
        errs = [ch for ch in checks if ch[0] == "error"]
        if errs:
            _expect_error(lambda: impl.matmul_q4_0(x, m, k, wb, n, k_in), errs[0][1])
            return
        out = np.asarray(impl.matmul_q4_0(x, m, k, wb, n, k_in))
        for ch in checks:
            if ch[0] == "shape":
                assert list(out.shape) == ch[1]
            elif ch[0] == "all_abs_lt":
                assert np.all(np.abs(out) < ch[1])
            elif ch[0] == "vs_dequant_naive_abs":
                wdeq = oracle.dequantize_q4_0(wb)
                ref = naive_matmul_t(x, wdeq, m, k, n)
                if hasattr(impl, "q4_close"):
                    # An implementation that reassociates the f32 sum states its
                    # own bound; the reference's 1e-5 absolute bound assumes the
                    # naive kernel's summation order.
                    assert impl.q4_close(out, ref, x.reshape(m, k), wdeq.reshape(n, k))
                else:
                    assert np.max(np.abs(out - ref)) < ch[1]
            else:
                raise KeyError(ch[0])
    elif op in ("dequantize_q8_0", "dequantize_q4_0"):
        data = np.array(c["data"], dtype=np.uint8)
        fn = getattr(impl, op)
        errs = [ch for ch in checks if ch[0] == "error"]
        if errs:
            _expect_error(lambda: fn(data), errs[0][1])
            return
        vals = np.asarray(fn(data))
        for ch in checks:
            if ch[0] == "values_approx":
                assert np.all(np.abs(vals - np.array(ch[1], dtype=np.float32)) < ch[2])
            elif ch[0] == "value_approx":
                assert abs(float(vals[ch[1]]) - ch[2]) < ch[3]
            else:
                raise KeyError(ch[0])
    elif op in ("create_q8_0_block", "create_q4_0_block"):
        v = np.array(c["values"], dtype=np.float32)
        blk = np.asarray(getattr(impl, op)(v))
        deq = impl.dequantize_q8_0 if op == "create_q8_0_block" else impl.dequantize_q4_0
        rec = np.asarray(deq(blk))
        for ch in checks:
            if ch[0] == "roundtrip_abs":
                if ch[1] == 0.0:
                    assert np.all(rec == 0.0)
                else:
                    assert np.all(np.abs(v - rec) < ch[1])
            elif ch[0] == "bytes_after_scale":
                assert np.all(blk[2:] == ch[1])
            else:
                raise KeyError(ch[0])
    elif op == "f16":
        for v in c["values"]:
            back = float(impl.f16_to_f32(impl.f32_to_f16(v)))
            assert abs(v - back) < abs(v) * 0.001 + 0.001, v
    elif op == "f16_specials":
        for bits, want in c["expect"]:
            got = float(impl.f16_to_f32(bits))
            if want == "nan":
                assert math.isnan(got)
            else:
                w = float(want)
                assert got == w and math.copysign(1.0, got) == math.copysign(1.0, w), (bits, got, want)
    else:
        raise KeyError(op)
