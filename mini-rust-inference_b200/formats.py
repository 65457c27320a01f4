"""Host-side weight formats: GGUF Q8_0 / Q4_0 block codecs and f16 bits.

Weight preparation happens once at load time on the host, as in the
reference (Q8_0WeightMatrix::from_f32_tensor, q8_direct.rs:118-158; the Q4_0
test packer, q4_0.rs:196-206).  These are vectorised numpy restatements of

  * gguf/dequant.rs:389-424  create_q8_0_block (f16 scale by the truncating
    f32_to_f16 of gguf/quantization.rs:464-498, quants from the f32 scale)
  * gguf/dequant.rs:706-749  create_q4_0_block (low nibble = even element)
  * gguf/quantization.rs:416-461 f16_to_f32 (exact IEEE half -> float)

The hot-path products never run here; they run in libmri_gpu.so.
"""
import numpy as np

Q8_0_BLOCK_BYTES = 34
Q4_0_BLOCK_BYTES = 18
BLOCK_ELEMS = 32


def f32_to_f16_trunc(values):
    """gguf/quantization.rs:464-498, bit for bit (mantissa truncated)."""
    f = np.ascontiguousarray(values, dtype=np.float32)
    bits = f.view(np.uint32).astype(np.int64)
    sign = (bits >> 31) & 1
    exp = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    s15 = sign << 15
    out = np.zeros(bits.shape, dtype=np.int64)
    normal = (exp >= 113) & (exp <= 142)
    out = np.where(normal, s15 | (((exp - 112) & 0x1F) << 10) | (mant >> 13), out)
    sub = (exp >= 103) & (exp < 113)
    shift = np.clip(126 - exp + 13, 0, 62)
    out = np.where(sub, s15 | ((mant | 0x800000) >> shift), out)
    out = np.where(exp < 103, s15, out)
    out = np.where((exp > 142) & (exp != 255), s15 | 0x7C00, out)
    nan_m = np.maximum(mant >> 13, 1)
    out = np.where(exp == 255, np.where(mant == 0, s15 | 0x7C00, s15 | 0x7C00 | nan_m), out)
    return out.astype(np.uint16)


def f16_to_f32(bits):
    """Exact half -> float (gguf/quantization.rs:416-461)."""
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def _round_half_away(x):
    """f32::round: half away from zero, exact in f32 (x - trunc(x) is exact)."""
    t = np.trunc(x)
    frac = x - t
    return np.where(np.abs(frac) >= np.float32(0.5), t + np.sign(x), t).astype(np.float32)


def _block_absmax(blocks):
    # fold(0.0, f32::max): NaN-skipping max starting at +0
    return np.fmax.reduce(np.abs(blocks), axis=-1, initial=np.float32(0.0)).astype(np.float32)


def quantize_q8_0(weights, n_out, k_in):
    """[n_out, k_in] f32 -> raw Q8_0 bytes (row-major blocks of 34 bytes)."""
    w = np.ascontiguousarray(weights, dtype=np.float32).reshape(n_out, k_in)
    if k_in % BLOCK_ELEMS:
        raise ValueError(f"k_in={k_in} not a multiple of 32")
    blocks = w.reshape(n_out, k_in // BLOCK_ELEMS, BLOCK_ELEMS)
    max_abs = _block_absmax(blocks)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        scale = np.where(max_abs == 0, np.float32(0.0), max_abs / np.float32(127.0)).astype(np.float32)
        inv = np.where(scale > 0, np.float32(1.0) / scale, np.float32(0.0)).astype(np.float32)
        r = _round_half_away(blocks * inv[..., None])
    q = np.where(np.isnan(r), 0, np.clip(r, -128, 127))
    q = np.where(scale[..., None] > 0, q, 0).astype(np.int8)
    out = np.empty((n_out, k_in // BLOCK_ELEMS, Q8_0_BLOCK_BYTES), dtype=np.uint8)
    out[..., 0:2] = f32_to_f16_trunc(scale).view(np.uint8).reshape(n_out, -1, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quantize_q4_0(weights, n_out, k):
    """[n_out, k] f32 -> raw Q4_0 bytes (row-major blocks of 18 bytes)."""
    w = np.ascontiguousarray(weights, dtype=np.float32).reshape(n_out, k)
    if k % BLOCK_ELEMS:
        raise ValueError(f"k={k} not a multiple of 32")
    blocks = w.reshape(n_out, k // BLOCK_ELEMS, BLOCK_ELEMS)
    max_abs = _block_absmax(blocks)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        scale = np.where(max_abs == 0, np.float32(0.0), max_abs / np.float32(7.0)).astype(np.float32)
        inv = np.where(scale > 0, np.float32(1.0) / scale, np.float32(0.0)).astype(np.float32)
        r = _round_half_away(blocks * inv[..., None])
    qi = np.where(np.isnan(r), 0, np.clip(r, -2.0 ** 31, 2.0 ** 31 - 1)).astype(np.int64)
    q = np.clip(qi + 8, 0, 15).astype(np.uint8)
    q = np.where(scale[..., None] > 0, q, 8).astype(np.uint8)
    out = np.empty((n_out, k // BLOCK_ELEMS, Q4_0_BLOCK_BYTES), dtype=np.uint8)
    out[..., 0:2] = f32_to_f16_trunc(scale).view(np.uint8).reshape(n_out, -1, 2)
    out[..., 2:] = q[..., 0::2] | (q[..., 1::2] << 4)
    return out.reshape(-1)


def dequantize_q8_0(data):
    """gguf/dequant.rs:103-133 (host; for tests and inspection)."""
    d = np.ascontiguousarray(data, dtype=np.uint8)
    if d.size % Q8_0_BLOCK_BYTES:
        raise ValueError("length not a multiple of 34")
    b = d.reshape(-1, Q8_0_BLOCK_BYTES)
    scale = f16_to_f32(b[:, 0:2].copy().view(np.uint16).reshape(-1))
    return (scale[:, None] * b[:, 2:].view(np.int8).astype(np.float32)).reshape(-1)


def dequantize_q4_0(data):
    """gguf/dequant.rs:471-500 (host; for tests and inspection)."""
    d = np.ascontiguousarray(data, dtype=np.uint8)
    if d.size % Q4_0_BLOCK_BYTES:
        raise ValueError("length not a multiple of 18")
    b = d.reshape(-1, Q4_0_BLOCK_BYTES)
    scale = f16_to_f32(b[:, 0:2].copy().view(np.uint16).reshape(-1))
    lo = (b[:, 2:] & 0x0F).astype(np.int32) - 8
    hi = (b[:, 2:] >> 4).astype(np.int32) - 8
    q = np.stack([lo, hi], axis=-1).reshape(-1, 32).astype(np.float32)
    return (scale[:, None] * q).reshape(-1)


def rope_table(max_seq, head_dim, base=10000.0):
    """RopeTable::new (ops/rope.rs:43-76): cos/sin [max_seq, head_dim/2] of
    pos * base^(-2i/head_dim), evaluated in f64 and rounded to f32."""
    half = head_dim // 2
    i = np.arange(half, dtype=np.float64)
    theta = 1.0 / np.power(np.float64(base), 2.0 * i / head_dim)
    ang = np.arange(max_seq, dtype=np.float64)[:, None] * theta[None, :]
    return np.cos(ang).astype(np.float32).reshape(-1), np.sin(ang).astype(np.float32).reshape(-1)
