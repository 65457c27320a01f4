"""The allocation-free entry point (mri_matmul_int8_from_f32_noalloc).

It exists for callers that cannot allocate device memory at call time: its
scratch is a fixed device array inside the library instead of a context's
growing buffer.  Through the C ABI it must agree with the regular entry point
(mri_matmul_int8_from_f32) bit for bit, on consecutive calls that reuse the
same scratch, on each of its paths (the streaming GEMV with the input
quantized in its prologue, the GEMV after quantizing a long input into the
array, the tensor-core GEMM), leave its sticky status word clear, and reject
inputs larger than the array.

This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run_pair(mri, lib, ctx, m, n, k, x_scale, seed):
    import torch
    rng = np.random.default_rng(seed)
    x = (rng.normal(0, 1, size=(m, k)) * x_scale).astype(np.float32)
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    qm = mri.QuantizedMatrix(wq, ws, n, k, ctx=ctx)
    xd = torch.from_numpy(x).cuda()
    wd = torch.from_numpy(wq).cuda()
    sd = torch.from_numpy(ws).cuda()
    out_ref = torch.empty(m, n, device="cuda")
    out_na = torch.full((m, n), float("nan"), device="cuda")
    rc = lib.mri_matmul_int8_from_f32(ctx.handle, ctypes.c_void_p(xd.data_ptr()), m, k, qm.handle,
                                      ctypes.c_void_p(out_ref.data_ptr()))
    assert rc == 0, mri._lib.last_error()
    ctx.synchronize()
    stream = torch.cuda.current_stream()
    rc = lib.mri_matmul_int8_from_f32_noalloc(ctypes.c_void_p(xd.data_ptr()), m, k,
                                              ctypes.c_void_p(wd.data_ptr()), ctypes.c_void_p(sd.data_ptr()),
                                              n, ctypes.c_void_p(out_na.data_ptr()),
                                              ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, lib.mri_noalloc_last_error().decode()
    # No bounded wait gave up (this also synchronizes the stream).
    rc = lib.mri_noalloc_check_status(ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, lib.mri_noalloc_last_error().decode()
    a = out_ref.cpu().numpy().view(np.uint32)
    b = out_na.cpu().numpy().view(np.uint32)
    assert np.array_equal(a, b), f"m={m}: {np.count_nonzero(a != b)} of {a.size} outputs differ"


def test_noalloc_matches_regular_entry_on_consecutive_calls(mri):
    lib = mri._lib.load()
    ctx = mri.Context(0)
    # First call: large activations (big absmax).  Second call: smaller
    # activations and a different shape, so stale scratch contents (absmax or
    # quantized rows) from the first call would change the result.
    _run_pair(mri, lib, ctx, 512, 1024, 4096, 4.0, seed=1)
    _run_pair(mri, lib, ctx, 37, 520, 2048, 0.25, seed=2)


def test_noalloc_decode_rows_match_regular_entry(mri):
    """1 and 8 rows (streaming GEMV, input quantized in its prologue), then a
    long input (K = 28672, quantized into the array first), then one row
    again: each against the regular entry point."""
    lib = mri._lib.load()
    ctx = mri.Context(0)
    _run_pair(mri, lib, ctx, 1, 11008, 4096, 1.0, seed=3)
    _run_pair(mri, lib, ctx, 8, 1000, 4096, 3.0, seed=4)
    _run_pair(mri, lib, ctx, 1, 2048, 28672, 0.5, seed=5)
    _run_pair(mri, lib, ctx, 1, 300, 1024, 2.0, seed=6)


def test_noalloc_rejects_oversized_input(mri):
    import torch
    lib = mri._lib.load()
    cap = 4 << 20
    x = torch.zeros(1, device="cuda")
    # One row too many, and a size whose product m * k wraps around to a
    # small number in 64 bits (2^60 + 1 rows of 16).
    for m, k in ((cap // 1024 + 1, 1024), ((1 << 60) + 1, 16)):
        rc = lib.mri_matmul_int8_from_f32_noalloc(ctypes.c_void_p(x.data_ptr()), m, k,
                                                  ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                                  8, ctypes.c_void_p(x.data_ptr()), None)
        assert rc == 6  # MRI_ERR_INVALID_ARGUMENT, before any launch
        assert b"exceed the fixed scratch" in lib.mri_noalloc_last_error()
