"""ctypes/numpy binding of the CPU oracle (oracle/ref_hotpath.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py as the checker / CPU baseline.  The product package never
imports this module.  Each wrapper names the reference function it restates.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

OK, INVALID_SHAPE, SHAPE_MISMATCH = 0, 1, 2
_P = ctypes.c_void_p
_SZ = ctypes.c_size_t


def build(force=False):
    """Compile the oracle with its Makefile (g++, -ffp-contract=off)."""
    src = os.path.join(_HERE, "ref_hotpath.cpp")
    hdr = os.path.join(_HERE, "ref_hotpath.h")
    if (not force and os.path.exists(_LIB_PATH)
            and os.path.getmtime(_LIB_PATH) >= max(os.path.getmtime(src), os.path.getmtime(hdr))):
        return _LIB_PATH
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "oref_quantize_symmetric": (ctypes.c_float, [_P, _SZ, _P]),
            "oref_quantize_symmetric_rows": (None, [_P, _SZ, _SZ, _P, _P]),
            "oref_dequantize_symmetric": (None, [_P, _SZ, ctypes.c_float, _P]),
            "oref_quantize_per_channel": (None, [_P, _SZ, _SZ, _P, _P]),
            "oref_matmul_int8": (ctypes.c_int, [_P, _SZ, ctypes.c_float, _P, _P, _SZ, _SZ, _SZ, _P, _P]),
            "oref_matmul_int8_from_f32": (ctypes.c_int, [_P, _SZ, _SZ, _P, _P, _SZ, _SZ, _P]),
            "oref_dot_i8_avx2": (ctypes.c_int32, [_P, _P, _SZ]),
            "oref_dot_i8_scalar": (ctypes.c_int32, [_P, _P, _SZ]),
            "oref_matmul_int8_avx2": (ctypes.c_int, [_P, _SZ, ctypes.c_float, _P, _P, _SZ, _SZ, _SZ, _P]),
            "oref_matmul_int8_parallel": (ctypes.c_int, [_P, _SZ, ctypes.c_float, _P, _P, _SZ, _SZ, _SZ, _P,
                                                         ctypes.c_int, _P]),
            "oref_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "oref_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "oref_create_q8_0_block": (None, [_P, _P]),
            "oref_create_q4_0_block": (None, [_P, _P]),
            "oref_quantize_q8_0_matrix": (ctypes.c_int, [_P, _SZ, _SZ, _P]),
            "oref_quantize_q4_0_matrix": (ctypes.c_int, [_P, _SZ, _SZ, _P]),
            "oref_dequantize_q8_0": (ctypes.c_int, [_P, _SZ, _P]),
            "oref_dequantize_q4_0": (ctypes.c_int, [_P, _SZ, _P]),
            "oref_q8_0_check_raw": (ctypes.c_int, [_SZ, _SZ, _SZ]),
            "oref_matmul_q8_0_direct": (ctypes.c_int, [_P, _SZ, _SZ, _P, _SZ, _SZ, _P]),
            "oref_matmul_q4_0_dequant": (ctypes.c_int, [_P, _SZ, _SZ, _P, _SZ, _SZ, _SZ, _P]),
            "oref_hardware_threads": (ctypes.c_int, []),
            "oref_rmsnorm": (None, [_P, _SZ, _SZ, _P, ctypes.c_float, _P]),
            "oref_rope_table": (None, [_SZ, _SZ, ctypes.c_float, _P, _P]),
            "oref_rope_apply": (None, [_P, _SZ, _SZ, _SZ, _P, _P, _SZ]),
            "oref_gqa_causal_offset": (None, [_P, _P, _P, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _P]),
            "oref_swiglu": (None, [_P, _P, _SZ, _P]),
            "oref_smooth_weight": (None, [_SZ, _SZ, ctypes.c_float, _P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i8(a):
    return np.ascontiguousarray(a, dtype=np.int8)


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


class OracleError(Exception):
    def __init__(self, code):
        super().__init__({INVALID_SHAPE: "InvalidShape", SHAPE_MISMATCH: "ShapeMismatch"}.get(code, code))
        self.kind = {INVALID_SHAPE: "InvalidShape", SHAPE_MISMATCH: "ShapeMismatch"}.get(code, str(code))


def _check(code):
    if code != OK:
        raise OracleError(code)


# symmetric.rs:42-57
def quantize_symmetric(x):
    x = _f32(x).ravel()
    q = np.empty(x.size, dtype=np.int8)
    s = lib().oref_quantize_symmetric(_ptr(x), x.size, _ptr(q))
    return q, np.float32(s)


# q8_direct.rs:260-264 (per-row application)
def quantize_symmetric_rows(x, m, k):
    x = _f32(x).ravel()
    q = np.empty(m * k, dtype=np.int8)
    s = np.empty(m, dtype=np.float32)
    lib().oref_quantize_symmetric_rows(_ptr(x), m, k, _ptr(q), _ptr(s))
    return q, s


def dequantize_symmetric(q, scale):
    q = _i8(q).ravel()
    out = np.empty(q.size, dtype=np.float32)
    lib().oref_dequantize_symmetric(_ptr(q), q.size, ctypes.c_float(scale), _ptr(out))
    return out


# per_channel.rs:98-128
def quantize_per_channel(w, n_out, k_in):
    w = _f32(w).ravel()
    assert w.size == n_out * k_in, "weights.len() != n_out*k_in"
    data = np.empty(n_out * k_in, dtype=np.int8)
    scales = np.empty(n_out, dtype=np.float32)
    lib().oref_quantize_per_channel(_ptr(w), n_out, k_in, _ptr(data), _ptr(scales))
    return data, scales


# int8.rs:61-98 -> (out[m, n], acc[m, n])
def matmul_int8(act_q, act_scale, w_data, w_scales, n_out, k_in, m):
    act_q = _i8(act_q).ravel()
    w_data = _i8(w_data).ravel()
    w_scales = _f32(w_scales).ravel()
    out = np.empty((m, n_out), dtype=np.float32)
    acc = np.empty((m, n_out), dtype=np.int32)
    _check(lib().oref_matmul_int8(_ptr(act_q), act_q.size, ctypes.c_float(act_scale), _ptr(w_data),
                                  _ptr(w_scales), n_out, k_in, m, _ptr(out), _ptr(acc)))
    return out, acc


# int8.rs:113-143
def matmul_int8_from_f32(x, m, k, w_data, w_scales, n_out, k_in):
    x = _f32(x).ravel()
    out = np.empty((m, n_out), dtype=np.float32)
    _check(lib().oref_matmul_int8_from_f32(_ptr(x), m, k, _ptr(_i8(w_data)), _ptr(_f32(w_scales)),
                                           n_out, k_in, _ptr(out)))
    return out


def dot_i8_avx2(a, b):
    a, b = _i8(a), _i8(b)
    return int(lib().oref_dot_i8_avx2(_ptr(a), _ptr(b), a.size))


def dot_i8_scalar(a, b):
    a, b = _i8(a), _i8(b)
    return int(lib().oref_dot_i8_scalar(_ptr(a), _ptr(b), a.size))


def matmul_int8_avx2(act_q, act_scale, w_data, w_scales, n_out, k_in, m):
    act_q = _i8(act_q).ravel()
    out = np.empty((m, n_out), dtype=np.float32)
    _check(lib().oref_matmul_int8_avx2(_ptr(act_q), act_q.size, ctypes.c_float(act_scale),
                                       _ptr(_i8(w_data)), _ptr(_f32(w_scales)), n_out, k_in, m, _ptr(out)))
    return out


# parallel.rs:308-346.  acc_out (optional int32 [m, n_out]) receives the dots
# before the epilogue (a checker's addition, for INT32 comparisons at sizes
# the scalar matmul_int8 is too slow for).
def matmul_int8_parallel(act_q, act_scale, w_data, w_scales, n_out, k_in, m, n_threads=0, out=None,
                         acc_out=None):
    act_q = _i8(act_q).ravel()
    if out is None:
        out = np.empty((m, n_out), dtype=np.float32)
    if acc_out is not None:
        assert acc_out.dtype == np.int32 and acc_out.size == m * n_out and acc_out.flags["C_CONTIGUOUS"]
    _check(lib().oref_matmul_int8_parallel(_ptr(act_q), act_q.size, ctypes.c_float(act_scale),
                                           _ptr(_i8(w_data)), _ptr(_f32(w_scales)), n_out, k_in, m,
                                           _ptr(out), int(n_threads), _ptr(acc_out)))
    return out


def f16_to_f32(h):
    return np.float32(lib().oref_f16_to_f32(int(h)))


def f32_to_f16(f):
    return int(lib().oref_f32_to_f16(ctypes.c_float(f)))


def create_q8_0_block(values32):
    v = _f32(values32)
    out = np.empty(34, dtype=np.uint8)
    lib().oref_create_q8_0_block(_ptr(v), _ptr(out))
    return out


def create_q4_0_block(values32):
    v = _f32(values32)
    out = np.empty(18, dtype=np.uint8)
    lib().oref_create_q4_0_block(_ptr(v), _ptr(out))
    return out


def quantize_q8_0_matrix(w, n_out, k_in):
    w = _f32(w).ravel()
    out = np.empty(n_out * (k_in // 32) * 34, dtype=np.uint8)
    _check(lib().oref_quantize_q8_0_matrix(_ptr(w), n_out, k_in, _ptr(out)))
    return out


def quantize_q4_0_matrix(w, n_out, k_in):
    w = _f32(w).ravel()
    out = np.empty(n_out * (k_in // 32) * 18, dtype=np.uint8)
    _check(lib().oref_quantize_q4_0_matrix(_ptr(w), n_out, k_in, _ptr(out)))
    return out


def dequantize_q8_0(data):
    d = _u8(data)
    out = np.empty((d.size // 34) * 32, dtype=np.float32)
    if lib().oref_dequantize_q8_0(_ptr(d), d.size, _ptr(out)) != 0:
        raise OracleError("AlignmentError")
    return out


def dequantize_q4_0(data):
    d = _u8(data)
    out = np.empty((d.size // 18) * 32, dtype=np.float32)
    if lib().oref_dequantize_q4_0(_ptr(d), d.size, _ptr(out)) != 0:
        raise OracleError("AlignmentError")
    return out


_F16 = None


def _f16_table():
    """f16_to_f32 (quantization.rs:416-461) of all 65536 bit patterns."""
    global _F16
    if _F16 is None:
        _F16 = np.array([f16_to_f32(h) for h in range(65536)], dtype=np.float32)
    return _F16


# gguf/extract.rs:719-737: F32 / F16 / Q8_0 / Q4_0 tensor bytes -> f32 values
# (extract_f32_from_bytes :772-815, f16_to_f32 per element, dequantize_q8_0 /
# dequantize_q4_0, dequant.rs:103-133 / 471-506).
def extract(ggml_type, raw):
    d = _u8(raw)
    if ggml_type == 0:
        return d.view(np.float32).copy()
    if ggml_type == 1:
        return _f16_table()[d.view(np.uint16)]
    if ggml_type == 8:
        return dequantize_q8_0(d)
    if ggml_type == 2:
        return dequantize_q4_0(d)
    raise OracleError("TypeMismatch")


# forward_int8.rs:52-62 (quantize_tensor) over extract(): what from_loader
# keeps of each projection.
def quantize_tensor(ggml_type, raw, n_out, k_in):
    return quantize_per_channel(extract(ggml_type, raw), n_out, k_in)


def q8_0_check_raw(data_len, n_out, k_in):
    return lib().oref_q8_0_check_raw(data_len, n_out, k_in)


# q8_direct.rs:229-289
def matmul_q8_0_direct(x, m, k, w_bytes, n_out, k_in):
    x = _f32(x).ravel()
    out = np.empty((m, n_out), dtype=np.float32)
    _check(lib().oref_matmul_q8_0_direct(_ptr(x), m, k, _ptr(_u8(w_bytes)), n_out, k_in, _ptr(out)))
    return out


# q4_0.rs:94-181
def matmul_q4_0_dequant(x, m, k_x, w_bytes, n_out, k):
    x = _f32(x).ravel()
    w = _u8(w_bytes)
    out = np.empty((m, n_out), dtype=np.float32)
    _check(lib().oref_matmul_q4_0_dequant(_ptr(x), m, k_x, _ptr(w), w.size, n_out, k, _ptr(out)))
    return out


def hardware_threads():
    return int(lib().oref_hardware_threads())


# ── model glue (LlamaModelInt8 checker) ──────────────────────────────────────

def rmsnorm(x, d, w, eps):
    x = _f32(x).reshape(-1)
    out = np.empty_like(x)
    lib().oref_rmsnorm(_ptr(x), x.size // d, d, _ptr(_f32(w)), ctypes.c_float(eps), _ptr(out))
    return out


def rope_table(max_seq, head_dim, base):
    c = np.empty(max_seq * (head_dim // 2), np.float32)
    s = np.empty_like(c)
    lib().oref_rope_table(max_seq, head_dim, ctypes.c_float(base), _ptr(c), _ptr(s))
    return c, s


def rope_apply(x, seq, n_heads, head_dim, cos_t, sin_t, start_pos):
    x = np.array(x, dtype=np.float32, copy=True).reshape(-1)
    lib().oref_rope_apply(_ptr(x), seq, n_heads, head_dim, _ptr(_f32(cos_t)), _ptr(_f32(sin_t)), start_pos)
    return x


def gqa_causal_offset(q, k, v, seq_q, seq_k, n_heads, n_kv, head_dim, start_pos):
    out = np.empty(seq_q * n_heads * head_dim, np.float32)
    lib().oref_gqa_causal_offset(_ptr(_f32(q)), _ptr(_f32(k)), _ptr(_f32(v)), seq_q, seq_k, n_heads, n_kv,
                                 head_dim, start_pos, _ptr(out))
    return out


def swiglu(gate, up):
    g, u = _f32(gate).reshape(-1), _f32(up).reshape(-1)
    out = np.empty_like(g)
    lib().oref_swiglu(_ptr(g), _ptr(u), g.size, _ptr(out))
    return out


def smooth_weight(rows, cols, seed):
    out = np.empty(rows * cols, np.float32)
    lib().oref_smooth_weight(rows, cols, ctypes.c_float(seed), _ptr(out))
    return out
