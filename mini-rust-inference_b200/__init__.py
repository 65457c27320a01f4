"""mini-rust-inference B200: the quantized-matmul hot path on sm_100a.

Host-side mirror of the reference's operator API (Rust crate
`llm-inference-engine`, module `ops::matmul` and `quant::int8`), backed by the
C ABI of libmri_gpu.so (include/mri_gpu.h).  Names, argument meaning and error
classes follow the reference:

  quantize_symmetric(values)                 quant/int8/symmetric.rs:42
  quantize_per_channel(weights, n_out, k_in) quant/int8/per_channel.rs:98
  matmul_int8(act_q, act_scale, weights, m)  ops/matmul/int8.rs:61
  matmul_int8_from_f32(input, weights)       ops/matmul/int8.rs:113
  matmul_int8_avx2 / _neon / _parallel       int8_avx2.rs:174, int8_neon.rs:158, parallel.rs:308
  matmul_q8_0_direct(input, weights)         ops/matmul/q8_direct.rs:229
  matmul_q4_0_dequant(input, w_q4, n_out, k) ops/matmul/q4_0.rs:94

Errors raise InvalidShape / ShapeMismatch (TensorError variants,
src/tensor/error.rs:7-29).  Inputs may be numpy arrays (host; synchronous
calls with H2D/D2H inside) or CUDA torch tensors (device; asynchronous on the
context's stream).  There is no CPU compute path.

Import with importlib (the directory name is not an identifier):
    mri = importlib.import_module("mini-rust-inference_b200")
"""
import contextlib
import ctypes
import sys
import threading

import numpy as np

from . import _lib
from . import formats

__all__ = [
    "TensorError", "InvalidShape", "ShapeMismatch", "CudaError", "DeviceTimeout",
    "Context", "default_context", "QuantizedMatrix", "Q8_0WeightMatrix", "Q4_0Matrix",
    "quantize_symmetric", "quantize_symmetric_rows", "quantize_per_channel",
    "matmul_int8", "matmul_int8_avx2", "matmul_int8_neon", "matmul_int8_parallel",
    "matmul_int8_from_f32", "matmul_q8_0_direct", "matmul_q4_0_dequant", "formats",
    "LlamaConfig", "LlamaModelInt8",
    "comm_available", "shard_rows", "Communicator", "shard_quantized_matrix",
    "matmul_int8_from_f32_sharded", "gguf_dequant",
]


# Activation-quantization granularity (mri_granularity).
PER_TENSOR, PER_ROW = _lib.PER_TENSOR, _lib.PER_ROW

# Kernel-variant options of a Context (mri_option in include/mri_gpu.h).
(OPT_PDL, OPT_GEMM_BN, OPT_GEMM_2CTA, OPT_Q8_MMA, OPT_Q4_MMA, OPT_TC_ATTN, OPT_FA_SPLIT, OPT_SHARD_PEER,
 OPT_GEMM_PAIR, OPT_Q4_LIMB) = range(10)


class TensorError(Exception):
    kind = "TensorError"


class InvalidShape(TensorError):
    kind = "InvalidShape"


class ShapeMismatch(TensorError):
    kind = "ShapeMismatch"


class CudaError(RuntimeError):
    kind = "CudaError"


class DeviceTimeout(RuntimeError):
    kind = "Timeout"


class CommError(RuntimeError):
    kind = "CommError"


_ERRORS = {
    _lib.INVALID_SHAPE: InvalidShape,
    _lib.SHAPE_MISMATCH: ShapeMismatch,
    _lib.CUDA_ERROR: CudaError,
    _lib.COMM_ERROR: CommError,
    _lib.TIMEOUT: DeviceTimeout,
    _lib.INVALID_ARGUMENT: ValueError,
}


def _check(rc):
    if rc != _lib.OK:
        raise _ERRORS.get(rc, RuntimeError)(_lib.last_error())


def _vp(arr):
    if arr is None:
        return None
    if isinstance(arr, np.ndarray):
        return arr.ctypes.data_as(ctypes.c_void_p)
    return ctypes.c_void_p(arr.data_ptr())


def _is_cuda_tensor(x):
    return hasattr(x, "is_cuda") and bool(getattr(x, "is_cuda"))


# ── contexts ──────────────────────────────────────────────────────────────────

class Context:
    """One CUDA stream + scratch on one device (mri_ctx)."""

    def __init__(self, device=0, stream=None):
        lib = _lib.load()
        h = ctypes.c_void_p()
        if stream is None:
            _check(lib.mri_ctx_create(int(device), ctypes.byref(h)))
        else:
            handle = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
            _check(lib.mri_ctx_create_on_stream(int(device), ctypes.c_void_p(handle), ctypes.byref(h)))
        self.handle = h
        self.device = int(device)
        self._lib = lib

    def close(self):
        if self.handle:
            self._lib.mri_ctx_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self, _finalizing=sys.is_finalizing):
        # At interpreter exit objects are finalized in no fixed order (a
        # context's stream may already be gone when a model or matrix that used
        # it is collected), and the process releases device memory anyway.
        # The check is bound at definition: module globals may be cleared by then.
        if _finalizing():
            return
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def synchronize(self):
        _check(self._lib.mri_ctx_synchronize(self.handle))

    def check_device_status(self):
        _check(self._lib.mri_ctx_check_device_status(self.handle))

    @property
    def launch_count(self):
        return int(self._lib.mri_ctx_launch_count(self.handle))

    @property
    def stream_handle(self):
        return int(self._lib.mri_ctx_stream(self.handle) or 0)

    def ordered_with_torch(self, device, launch):
        """Run `launch()`, which enqueues work on this context's stream, in
        order with torch's current stream on `device`: the context's stream
        first waits for what torch has queued (e.g. the copy that made an input
        contiguous), and torch's current stream then waits for the launched
        work, so torch consumers and torch's caching allocator see the outputs
        only once they are written.  The context's own stream is created
        non-blocking, so without these waits the two streams run unordered."""
        import torch
        cur = torch.cuda.current_stream(device)
        if cur.cuda_stream == self.stream_handle:
            return launch()
        ts = getattr(self, "_torch_stream", None)
        if ts is None:
            ts = self._torch_stream = torch.cuda.ExternalStream(self.stream_handle, device=device)
        ts.wait_stream(cur)
        try:
            return launch()
        finally:
            cur.wait_stream(ts)

    def int8_path(self, m, n, k):
        return int(self._lib.mri_int8_path(self.handle, m, n, k))

    def int8_gemv_plan(self, m, n, k):
        """Launch shape of the streaming INT8 GEMV (diagnostics)."""
        p = (ctypes.c_int * 8)()
        _check(self._lib.mri_int8_gemv_plan(self.handle, m, n, k, p))
        keys = ("grid", "ctas_per_sm", "resident_ctas", "stages", "k_chunks", "smem_bytes", "reg_vec",
                "quantize_first")
        return dict(zip(keys, list(p)))

    def int8_gemm_plan(self, m, n, k):
        """Launch shape of the tensor-core INT8 GEMM (diagnostics)."""
        p = (ctypes.c_int * 7)()
        _check(self._lib.mri_int8_gemm_plan(self.handle, m, n, k, p))
        keys = ("bn", "stages", "acc_buffers", "grid", "tiles", "tiles_per_cta", "cta_pair")
        return dict(zip(keys, list(p)))

    def set_option(self, option, value):
        """Kernel-variant option (OPT_* below; mri_ctx_set_option)."""
        _check(self._lib.mri_ctx_set_option(self.handle, int(option), int(value)))

    def get_option(self, option):
        v = ctypes.c_int()
        _check(self._lib.mri_ctx_get_option(self.handle, int(option), ctypes.byref(v)))
        return v.value

    @contextlib.contextmanager
    def option(self, option, value):
        """Sets an option for the body of a with-statement, then restores it."""
        old = self.get_option(option)
        self.set_option(option, value)
        try:
            yield self
        finally:
            self.set_option(option, old)


_tls = threading.local()


def default_context(device=0):
    """Per-thread, per-device context with its own stream."""
    ctxs = getattr(_tls, "ctxs", None)
    if ctxs is None:
        ctxs = _tls.ctxs = {}
    if device not in ctxs:
        ctxs[device] = Context(device)
    return ctxs[device]


def _ctx_for(ctx, x=None):
    if ctx is not None:
        return ctx
    dev = x.device.index if _is_cuda_tensor(x) else 0
    return default_context(dev or 0)


# ── weights ───────────────────────────────────────────────────────────────────

class QuantizedMatrix:
    """Device-resident QuantizedMatrix {data [n_out,k_in] i8, scales [n_out] f32}
    (quant/int8/per_channel.rs:29-40).  `rows=(begin, end)` uploads only that
    row range (an N-shard)."""

    def __init__(self, data, scales, n_out, k_in, ctx=None, rows=None, keep_host=True):
        self.ctx = ctx or default_context()
        data = np.ascontiguousarray(data, dtype=np.int8).reshape(-1)
        scales = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
        if data.size != n_out * k_in or scales.size != n_out:
            raise InvalidShape(f"QuantizedMatrix: data.len()={data.size}, scales.len()={scales.size} "
                               f"for n_out={n_out}, k_in={k_in}")
        begin, end = rows if rows is not None else (0, n_out)
        h = ctypes.c_void_p()
        _check(self.ctx._lib.mri_qmatrix_upload_rows(self.ctx.handle, _vp(data), _vp(scales), n_out,
                                                     k_in, begin, end, ctypes.byref(h)))
        self.handle = h
        self.n_out = end - begin
        self.k_in = k_in
        self.row_range = (begin, end)
        if keep_host:
            self.data = data.reshape(n_out, k_in)[begin:end].reshape(-1)
            self.scales = scales[begin:end]

    def __del__(self, _finalizing=sys.is_finalizing):
        # At interpreter exit objects are finalized in no fixed order (a
        # context's stream may already be gone when a model or matrix that used
        # it is collected), and the process releases device memory anyway.
        # The check is bound at definition: module globals may be cleared by then.
        if _finalizing():
            return
        try:
            if self.handle:
                self.ctx._lib.mri_qmatrix_free(self.handle)
        except Exception:  # noqa: BLE001
            pass

    @classmethod
    def from_gguf(cls, ggml_type, raw, n_out, k_in, ctx=None, keep_host=True):
        """quantize_tensor(&extractor.extract(name)) (forward_int8.rs:52-62,
        gguf/extract.rs:719-737) from a tensor's raw GGUF bytes: dequantized and
        requantized per row on the device, bit-identical to the host path."""
        self = cls.__new__(cls)
        self.ctx = ctx or default_context()
        raw = np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw
        raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
        h = ctypes.c_void_p()
        self.handle = None
        _check(self.ctx._lib.mri_qmatrix_from_gguf(self.ctx.handle, int(ggml_type), _vp(raw), raw.size,
                                                   n_out, k_in, ctypes.byref(h)))
        self.handle = h
        self.n_out, self.k_in, self.row_range = n_out, k_in, (0, n_out)
        if keep_host:
            self.data = np.empty(n_out * k_in, np.int8)
            self.scales = np.empty(n_out, np.float32)
            _check(self.ctx._lib.mri_qmatrix_download(h, _vp(self.data), _vp(self.scales)))
        return self

    def row(self, n):
        """per_channel.rs:45-48"""
        return self.data[n * self.k_in:(n + 1) * self.k_in]

    def dequantize_row(self, n):
        return self.row(n).astype(np.float32) * self.scales[n]

    def dequantize_all(self):
        return (self.data.reshape(self.n_out, self.k_in).astype(np.float32) * self.scales[:, None]).reshape(-1)


class Q8_0WeightMatrix:
    """Device-resident raw Q8_0 bytes (ops/matmul/q8_direct.rs:60-197)."""

    def __init__(self, handle, data, n_out, k_in, ctx):
        self.handle, self.data, self.n_out, self.k_in, self.ctx = handle, data, n_out, k_in, ctx
        self.n_blocks = k_in // 32

    @classmethod
    def from_raw_bytes(cls, data, n_out, k_in, ctx=None):
        """q8_direct.rs:80-107 (InvalidShape on k % 32 or byte length)."""
        ctx = ctx or default_context()
        d = np.frombuffer(bytes(data), dtype=np.uint8) if isinstance(data, (bytes, bytearray)) \
            else np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
        h = ctypes.c_void_p()
        _check(ctx._lib.mri_q8_0_upload(ctx.handle, _vp(d), d.size, n_out, k_in, ctypes.byref(h)))
        return cls(h, d, n_out, k_in, ctx)

    @classmethod
    def from_f32_tensor(cls, t, ctx=None):
        """q8_direct.rs:118-158"""
        t = np.asarray(t, dtype=np.float32)
        if t.ndim != 2:
            raise InvalidShape(f"Q8_0WeightMatrix::from_f32_tensor: expected 2-D, got {t.ndim}D")
        n_out, k_in = t.shape
        if k_in % 32:
            raise InvalidShape(f"Q8_0WeightMatrix::from_f32_tensor: k_in={k_in} not a multiple of 32")
        return cls.from_raw_bytes(formats.quantize_q8_0(t, n_out, k_in), n_out, k_in, ctx)

    def block_scale(self, n, b):
        off = (n * self.n_blocks + b) * 34
        return formats.f16_to_f32(self.data[off:off + 2].copy().view(np.uint16))[0]

    def dequantize_all(self):
        return formats.dequantize_q8_0(self.data)

    def __del__(self, _finalizing=sys.is_finalizing):
        # At interpreter exit objects are finalized in no fixed order (a
        # context's stream may already be gone when a model or matrix that used
        # it is collected), and the process releases device memory anyway.
        # The check is bound at definition: module globals may be cleared by then.
        if _finalizing():
            return
        try:
            if self.handle:
                self.ctx._lib.mri_q8_0_free(self.handle)
        except Exception:  # noqa: BLE001
            pass


class Q4_0Matrix:
    """Device-resident Q4_0 bytes of a [n_out, k] weight (q4_0.rs:8-21)."""

    def __init__(self, data, n_out, k, ctx=None):
        self.ctx = ctx or default_context()
        d = np.frombuffer(bytes(data), dtype=np.uint8) if isinstance(data, (bytes, bytearray)) \
            else np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
        h = ctypes.c_void_p()
        _check(self.ctx._lib.mri_q4_0_upload(self.ctx.handle, _vp(d), d.size, n_out, k, ctypes.byref(h)))
        self.handle, self.data, self.n_out, self.k = h, d, n_out, k

    def __del__(self, _finalizing=sys.is_finalizing):
        # At interpreter exit objects are finalized in no fixed order (a
        # context's stream may already be gone when a model or matrix that used
        # it is collected), and the process releases device memory anyway.
        # The check is bound at definition: module globals may be cleared by then.
        if _finalizing():
            return
        try:
            if self.handle:
                self.ctx._lib.mri_q4_0_free(self.handle)
        except Exception:  # noqa: BLE001
            pass


# ── quantizers ────────────────────────────────────────────────────────────────

def gguf_dequant(ggml_type, raw, numel, out=None, ctx=None):
    """TensorExtractor::extract (gguf/extract.rs:719-737) of a tensor's raw GGUF
    bytes, dequantized on the device: `out` (a CUDA float32 tensor of numel
    values) is filled, or a host float32 array is returned."""
    ctx = ctx or default_context()
    raw = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray)
                               else raw, dtype=np.uint8).reshape(-1)
    if out is not None:
        ctx.ordered_with_torch(out.device, lambda: _check(ctx._lib.mri_gguf_dequant(
            ctx.handle, int(ggml_type), _vp(raw), raw.size, numel, _vp(out))))
        ctx.synchronize()
        return out
    import torch
    dev = torch.empty(max(numel, 1), dtype=torch.float32, device=f"cuda:{ctx.device}")
    _check(ctx._lib.mri_gguf_dequant(ctx.handle, int(ggml_type), _vp(raw), raw.size, numel, _vp(dev)))
    ctx.synchronize()
    return dev[:numel].cpu().numpy()


def _host_quantize(values, m, k, granularity, ctx):
    ctx = ctx or default_context()
    x = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    q = np.empty(m * k, dtype=np.int8)
    s = np.empty(max(m, 1) if granularity == _lib.PER_ROW else 1, dtype=np.float32)
    _check(ctx._lib.mri_host_quantize_symmetric(ctx.handle, _vp(x), m, k, granularity, _vp(q), _vp(s)))
    return q, s


def quantize_symmetric(values, ctx=None):
    """symmetric.rs:42-57 -> (q: int8[len], scale: float32)."""
    v = np.asarray(values, dtype=np.float32).reshape(-1)
    q, s = _host_quantize(v, 1, v.size, _lib.PER_TENSOR, ctx)
    return q, np.float32(s[0])


def quantize_symmetric_rows(values, m, k, ctx=None):
    """quantize_symmetric applied to each row (q8_direct.rs:260-264)."""
    q, s = _host_quantize(values, m, k, _lib.PER_ROW, ctx)
    return q, s[:m]


def quantize_per_channel(weights, n_out, k_in, ctx=None, rows=None):
    """per_channel.rs:98-128, run on the GPU (per-row absmax quantization has
    the same formula), returning the device-resident matrix."""
    w = np.asarray(weights, dtype=np.float32).reshape(-1)
    assert w.size == n_out * k_in, f"weights.len()={w.size} != n_out*k_in={n_out * k_in}"
    q, s = _host_quantize(w, n_out, k_in, _lib.PER_ROW, ctx)
    return QuantizedMatrix(q, s[:n_out], n_out, k_in, ctx=ctx, rows=rows)


# ── products ──────────────────────────────────────────────────────────────────

def _as_2d(input_, fn):
    if _is_cuda_tensor(input_):
        if input_.dim() != 2:
            raise InvalidShape(f"{fn}: input must be 2-D, got {input_.dim()}D (shape {list(input_.shape)})")
        return input_.contiguous()
    a = np.asarray(input_, dtype=np.float32)
    if a.ndim != 2:
        raise InvalidShape(f"{fn}: input must be 2-D, got {a.ndim}D (shape {list(a.shape)})")
    return np.ascontiguousarray(a)


def _new_out(like, m, n):
    if _is_cuda_tensor(like):
        import torch
        return torch.empty((m, n), dtype=torch.float32, device=like.device)
    return np.empty((m, n), dtype=np.float32)


def matmul_int8(act_q, act_scale, weights, m, acc_out=None):
    """ops/matmul/int8.rs:61-98.  Returns f32 [m, n]; `acc_out` (optional,
    int32 [m, n], same residency as act_q) receives the INT32 accumulators."""
    ctx = weights.ctx
    n = weights.n_out
    if _is_cuda_tensor(act_q):
        act_q = act_q.contiguous()
        out = _new_out(act_q, m, n)
        ctx.ordered_with_torch(act_q.device, lambda: _check(ctx._lib.mri_matmul_int8(
            ctx.handle, _vp(act_q), act_q.numel(), float(act_scale), weights.handle, m, _vp(out),
            _vp(acc_out))))
        return out
    a = np.ascontiguousarray(act_q, dtype=np.int8).reshape(-1)
    out = np.empty((m, n), dtype=np.float32)
    _check(ctx._lib.mri_host_matmul_int8(ctx.handle, _vp(a), a.size, float(act_scale), weights.handle,
                                         m, _vp(out), _vp(acc_out)))
    return out


# One GPU kernel serves every reference variant (scalar, AVX2, NEON, rayon).
matmul_int8_avx2 = matmul_int8
matmul_int8_neon = matmul_int8
matmul_int8_parallel = matmul_int8


def matmul_int8_from_f32(input, weights, granularity=_lib.PER_TENSOR):  # noqa: A002 - reference name
    """ops/matmul/int8.rs:113-143 (per-tensor activation scale by default)."""
    x = _as_2d(input, "matmul_int8_from_f32")
    m, k = x.shape
    if k != weights.k_in:
        raise ShapeMismatch(f"expected [{m}, {weights.k_in}], got [{m}, {k}]")
    ctx = weights.ctx
    out = _new_out(x, m, weights.n_out)
    if _is_cuda_tensor(x):
        ctx.ordered_with_torch(x.device, lambda: _check(ctx._lib.mri_matmul_int8_from_f32_g(
            ctx.handle, _vp(x), m, k, granularity, weights.handle, _vp(out))))
    elif granularity == _lib.PER_TENSOR:
        _check(ctx._lib.mri_host_matmul_int8_from_f32(ctx.handle, _vp(x), m, k, weights.handle, _vp(out)))
    else:
        q, s = quantize_symmetric_rows(x, m, k, ctx)
        import torch  # per-row host path goes through device buffers
        dq = torch.from_numpy(q).cuda(ctx.device)
        ds = torch.from_numpy(s).cuda(ctx.device)
        dout = torch.empty((m, weights.n_out), dtype=torch.float32, device=f"cuda:{ctx.device}")
        _check(ctx._lib.mri_matmul_int8_dscale(ctx.handle, _vp(dq), m * k, _vp(ds), 1, weights.handle,
                                               m, _vp(dout), None))
        ctx.synchronize()
        out = dout.cpu().numpy()
    return out


def matmul_q8_0_direct(input, weights):  # noqa: A002
    """ops/matmul/q8_direct.rs:229-289 (bit-exact)."""
    x = _as_2d(input, "matmul_q8_0_direct")
    m, k = x.shape
    if k != weights.k_in:
        raise ShapeMismatch(f"expected [{m}, {weights.k_in}], got [{m}, {k}]")
    ctx = weights.ctx
    out = _new_out(x, m, weights.n_out)
    if _is_cuda_tensor(x):
        ctx.ordered_with_torch(x.device, lambda: _check(ctx._lib.mri_matmul_q8_0_direct(
            ctx.handle, _vp(x), m, k, weights.handle, _vp(out))))
    else:
        _check(ctx._lib.mri_host_matmul_q8_0_direct(ctx.handle, _vp(x), m, k, weights.handle, _vp(out)))
    return out


def matmul_q4_0_dequant(input, weight_q4, n_out, k, ctx=None):  # noqa: A002
    """ops/matmul/q4_0.rs:94-181.  `weight_q4` is the raw byte slice (uploaded
    for this call) or a Q4_0Matrix already on the device.  Checks run in the
    reference's order: 2-D, K mismatch, k % 32, byte length."""
    x = _as_2d(input, "matmul_q4_0_dequant")
    m, k_in = x.shape
    if k_in != k:
        raise ShapeMismatch(f"expected [{m}, {k}], got [{m}, {k_in}]")
    w = weight_q4 if isinstance(weight_q4, Q4_0Matrix) else Q4_0Matrix(weight_q4, n_out, k, ctx=ctx)
    if (w.n_out, w.k) != (n_out, k):
        raise InvalidShape(f"Q4_0Matrix is [{w.n_out}, {w.k}], call says [{n_out}, {k}]")
    c = w.ctx
    out = _new_out(x, m, n_out)
    if _is_cuda_tensor(x):
        c.ordered_with_torch(x.device, lambda: _check(c._lib.mri_matmul_q4_0_dequant(
            c.handle, _vp(x), m, k, w.handle, _vp(out))))
    else:
        _check(c._lib.mri_host_matmul_q4_0_dequant(c.handle, _vp(x), m, k, w.handle, _vp(out)))
    return out


def library_path():
    return _lib.library_path()


# ── N-sharded products (no reference counterpart) ─────────────────────────────

def comm_available():
    """True when libnccl.so.2 could be loaded by the library."""
    return bool(_lib.load().mri_comm_available())


def shard_rows(n, nranks, rank):
    """Rows [begin, end) of an [n, k] weight that rank `rank` of `nranks` holds
    (equal shards; InvalidShape when n % nranks != 0)."""
    lib = _lib.load()
    b, e = ctypes.c_size_t(), ctypes.c_size_t()
    _check(lib.mri_shard_rows(int(n), int(nranks), int(rank), ctypes.byref(b), ctypes.byref(e)))
    return b.value, e.value


class Communicator:
    """NCCL communicator bound to one context (mri_comm).  One per rank; rank
    0's `unique_id()` bytes must reach every rank before construction."""

    ID_BYTES = 128

    @staticmethod
    def unique_id():
        buf = (ctypes.c_uint8 * Communicator.ID_BYTES)()
        _check(_lib.load().mri_comm_unique_id(buf))
        return bytes(buf)

    def __init__(self, unique_id, nranks, rank, ctx=None, timeout_ms=60000):
        self.ctx = ctx or default_context()
        if len(unique_id) != self.ID_BYTES:
            raise ValueError(f"unique id must be {self.ID_BYTES} bytes")
        buf = (ctypes.c_uint8 * self.ID_BYTES).from_buffer_copy(unique_id)
        h = ctypes.c_void_p()
        _check(self.ctx._lib.mri_comm_create(self.ctx.handle, buf, int(nranks), int(rank), int(timeout_ms),
                                             ctypes.byref(h)))
        self.handle = h
        self.rank, self.size = int(rank), int(nranks)

    @classmethod
    def from_process_group(cls, ctx=None, group=None, timeout_ms=60000):
        """Rendezvous over an initialised torch.distributed group (rank 0's id
        broadcast with broadcast_object_list)."""
        import torch.distributed as dist
        obj = [cls.unique_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(obj[0], dist.get_world_size(group), dist.get_rank(group), ctx=ctx, timeout_ms=timeout_ms)

    def wait(self):
        _check(self.ctx._lib.mri_comm_wait(self.handle))

    def close(self):
        if self.handle:
            self.ctx._lib.mri_comm_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self, _finalizing=sys.is_finalizing):
        # At interpreter exit objects are finalized in no fixed order (a
        # context's stream may already be gone when a model or matrix that used
        # it is collected), and the process releases device memory anyway.
        # The check is bound at definition: module globals may be cleared by then.
        if _finalizing():
            return
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def shard_quantized_matrix(data, scales, n_out, k_in, comm, keep_host=False):
    """Upload this rank's N-shard (shard_rows) of a QuantizedMatrix."""
    return QuantizedMatrix(data, scales, n_out, k_in, ctx=comm.ctx,
                           rows=shard_rows(n_out, comm.size, comm.rank), keep_host=keep_host)


def matmul_int8_from_f32_sharded(input, w_shard, n_total, comm):  # noqa: A002
    """matmul_int8_from_f32 (ops/matmul/int8.rs:113-143) of the full weight
    whose rows are split across the communicator's ranks: every rank gets the
    full [m, n_total] product.  Device tensors in -> device tensor out
    (asynchronous); host arrays -> host array (synchronous)."""
    x = _as_2d(input, "matmul_int8_from_f32_sharded")
    m, k = x.shape
    lib = comm.ctx._lib
    if _is_cuda_tensor(x):
        out = _new_out(x, m, n_total)
        comm.ctx.ordered_with_torch(x.device, lambda: _check(lib.mri_sharded_matmul_int8_from_f32(
            comm.handle, _vp(x), m, k, w_shard.handle, n_total, _vp(out))))
        return out
    import torch
    dev = f"cuda:{comm.ctx.device}"
    dx = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    dout = torch.empty((m, n_total), dtype=torch.float32, device=dev)
    torch.cuda.synchronize(comm.ctx.device)
    _check(lib.mri_sharded_matmul_int8_from_f32(comm.handle, _vp(dx), m, k, w_shard.handle, n_total,
                                                _vp(dout)))
    comm.wait()
    return dout.cpu().numpy()


# ── LlamaModelInt8 (model/llama/forward_int8.rs:416-547) ─────────────────────

class LlamaConfig(ctypes.Structure):
    """Mirror of LlamaConfig (model/llama/config.rs:31-52), the fields the INT8
    forward pass uses; n_kv_heads = 0 means n_heads."""
    _fields_ = [("n_layers", ctypes.c_uint32), ("dim", ctypes.c_uint32), ("n_heads", ctypes.c_uint32),
                ("n_kv_heads", ctypes.c_uint32), ("ffn_dim", ctypes.c_uint32), ("vocab", ctypes.c_uint32),
                ("max_seq", ctypes.c_uint32), ("rope_base", ctypes.c_float), ("rms_eps", ctypes.c_float)]

    def __init__(self, n_layers, dim, n_heads, ffn_dim, vocab, max_seq, n_kv_heads=0,
                 rope_base=10000.0, rms_eps=1e-5):
        super().__init__(n_layers, dim, n_heads, n_kv_heads, ffn_dim, vocab, max_seq, rope_base, rms_eps)

    @property
    def head_dim(self):
        return self.dim // self.n_heads

    @property
    def kv_heads(self):
        return self.n_kv_heads or self.n_heads


def _check_model(rc, lib):
    if rc != _lib.OK:
        raise _ERRORS.get(rc, RuntimeError)(lib.mri_llama_last_error().decode(errors="replace"))


class LlamaModelInt8:
    """Device-resident LlamaModelInt8.  Build with `from_weights` (host arrays,
    as LlamaModelInt8::new takes pre-quantized blocks) or `random` (synthetic
    weights generated on the GPU, for benchmarks)."""

    def __init__(self, cfg, ctx=None):
        self.ctx = ctx or default_context()
        self.cfg = cfg
        self._lib = self.ctx._lib
        h = ctypes.c_void_p()
        _check_model(self._lib.mri_llama_create(self.ctx.handle, ctypes.byref(cfg), ctypes.byref(h)), self._lib)
        self.handle = h

    def __del__(self, _finalizing=sys.is_finalizing):
        # At interpreter exit objects are finalized in no fixed order (a
        # context's stream may already be gone when a model or matrix that used
        # it is collected), and the process releases device memory anyway.
        # The check is bound at definition: module globals may be cleared by then.
        if _finalizing():
            return
        try:
            if self.handle:
                self._lib.mri_llama_free(self.handle)
        except Exception:  # noqa: BLE001
            pass

    def set_rope(self, cos_t=None, sin_t=None):
        if cos_t is None:
            cos_t, sin_t = formats.rope_table(self.cfg.max_seq, self.cfg.head_dim, self.cfg.rope_base)
        c, s = np.ascontiguousarray(cos_t, np.float32), np.ascontiguousarray(sin_t, np.float32)
        _check_model(self._lib.mri_llama_set_rope(self.handle, _vp(c), _vp(s)), self._lib)

    @classmethod
    def from_weights(cls, cfg, w, ctx=None, rope=None):
        """w: dict with token_embd [vocab*dim] f32, attn_norm/ffn_norm [L*dim],
        output_norm [dim], output (data, scales), and layers: list of dicts with
        wq, wk, wv, wo, wgate, wup, wdown each (int8 data, f32 scales)."""
        m = cls(cfg, ctx)
        lib = m._lib
        f32 = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
        i8 = lambda a: np.ascontiguousarray(a, np.int8)  # noqa: E731
        keep = []
        _check_model(lib.mri_llama_set_embedding(m.handle, _vp(f32(w["token_embd"]))), lib)
        an, fn, on = f32(w["attn_norm"]), f32(w["ffn_norm"]), f32(w["output_norm"])
        _check_model(lib.mri_llama_set_norms(m.handle, _vp(an), _vp(fn), _vp(on)), lib)
        for li, layer in enumerate(w["layers"]):
            args = []
            for name in ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown"):
                d, s = i8(layer[name][0]), f32(layer[name][1])
                keep += [d, s]
                args += [_vp(d), _vp(s)]
            _check_model(lib.mri_llama_set_layer(m.handle, li, *args), lib)
        od, os_ = i8(w["output"][0]), f32(w["output"][1])
        _check_model(lib.mri_llama_set_output(m.handle, _vp(od), _vp(os_)), lib)
        m.set_rope(*(rope or (None, None)))
        return m

    @classmethod
    def from_gguf(cls, path, ctx=None, max_seq=None):
        """LlamaModelInt8::from_loader (forward_int8.rs:461-507): configuration
        from the file's metadata (LlamaConfig::from_metadata), every tensor's
        raw bytes from the mapped file to the device, projections requantized
        per channel there, embedding and norms dequantized to f32 there.
        `max_seq` (default: llama.context_length) sizes the KV cache and the
        RoPE table.  Raises gguf.MissingMetadataKey / InvalidConfig /
        KeyNotFound / TensorDataUnavailable, or the ABI's errors."""
        from . import gguf
        g = path if isinstance(path, gguf.GgufFile) else gguf.GgufFile(path)
        c = gguf.llama_config(g.metadata)
        cfg = LlamaConfig(c["block_count"], c["embedding_length"], c["n_heads"], c["feed_forward_length"],
                          c["vocab_size"], int(max_seq or c["context_length"]), n_kv_heads=c["n_kv_heads"],
                          rope_base=c["rope_freq_base"], rms_eps=c["rms_norm_eps"])
        m = cls(cfg, ctx)
        lib = m._lib

        def load(name, role, layer):
            info = g.tensor(name)
            raw = g.tensor_data(name)
            if raw is None:
                raise gguf.TensorDataUnavailable(name)
            shape = info.shape_row_major()
            rows, cols = (1, shape[0]) if len(shape) == 1 else (int(np.prod(shape[:-1])), shape[-1])
            _check_model(lib.mri_llama_load_tensor(m.handle, role, layer, info.dtype, _vp(raw), raw.size,
                                                   rows, cols), lib)

        for name, role in gguf.GLOBAL_TENSORS:
            load(name, role, 0)
        for layer in range(cfg.n_layers):
            for suffix, role in gguf.LAYER_TENSORS:
                load(gguf.weight_name(layer, suffix), role, layer)
        m.set_rope()
        return m

    @classmethod
    def random(cls, cfg, seed=0, ctx=None):
        m = cls(cfg, ctx)
        _check_model(m._lib.mri_llama_init_random(m.handle, int(seed)), m._lib)
        m.set_rope()
        return m

    def forward(self, tokens):
        """forward_int8.rs:516-529: logits [len(tokens), vocab]."""
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.empty((t.size, self.cfg.vocab), np.float32)
        _check_model(self._lib.mri_llama_forward(self.handle, _vp(t), t.size, _vp(out)), self._lib)
        return out

    def forward_at(self, tokens, start_pos):
        """The block loop of TransformerBlockInt8::forward_cached_parallel
        (forward_int8.rs:232-249) at `start_pos`: the tokens take positions
        [start_pos, start_pos + len), write their K/V cache rows there and
        attend to the cache from row 0.  Logits [len(tokens), vocab]."""
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.empty((t.size, self.cfg.vocab), np.float32)
        _check_model(self._lib.mri_llama_forward_at(self.handle, _vp(t), t.size, int(start_pos), _vp(out)),
                     self._lib)
        return out

    def block_forward(self, layer, x, start_pos):
        """TransformerBlockInt8::forward_cached_parallel(x, start_pos, cache,
        layer) (forward_int8.rs:232-249) with the model's KV cache: x f32
        [n, dim] -> [n, dim]."""
        xa = np.ascontiguousarray(x, np.float32).reshape(-1, self.cfg.dim)
        out = np.empty_like(xa)
        _check_model(self._lib.mri_llama_block_forward(self.handle, int(layer), _vp(xa), xa.shape[0],
                                                       int(start_pos), _vp(out)), self._lib)
        return out

    def set_option(self, option, value):
        """A kernel-variant option (OPT_*) for this model alone."""
        _check_model(self._lib.mri_llama_set_option(self.handle, int(option), int(value)), self._lib)

    def attention_fallbacks(self):
        """Calls run again with the f32 prefill attention (q, k or v beyond
        the f16 range)."""
        n = ctypes.c_size_t()
        _check_model(self._lib.mri_llama_attention_fallbacks(self.handle, ctypes.byref(n)), self._lib)
        return n.value

    def forward_decode(self, token, pos):
        """forward_int8.rs:538-546: logits [vocab] for `token` at `pos` (the
        cache must hold positions [0, pos))."""
        out = np.empty(self.cfg.vocab, np.float32)
        _check_model(self._lib.mri_llama_forward_decode(self.handle, int(token), int(pos), _vp(out)), self._lib)
        return out

    def generate_greedy(self, prompt, n_decode):
        """Prefill + n_decode greedy steps; returns (tokens [n_decode+1],
        prefill_ms, decode_ms), device-timed."""
        p = np.ascontiguousarray(prompt, np.uint32)
        toks = np.empty(n_decode + 1, np.uint32)
        pm, dm = ctypes.c_float(), ctypes.c_float()
        _check_model(self._lib.mri_llama_generate_greedy(self.handle, _vp(p), p.size, n_decode, _vp(toks),
                                                         ctypes.byref(pm), ctypes.byref(dm)), self._lib)
        return toks, pm.value, dm.value

    def kernels_per_decode_step(self):
        n = ctypes.c_size_t()
        _check_model(self._lib.mri_llama_launches_per_decode_step(self.handle, ctypes.byref(n)), self._lib)
        return n.value
