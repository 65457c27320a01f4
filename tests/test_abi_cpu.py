"""CPU-only checks of the boundary: the C-ABI library loads, exports every
symbol include/*.h declares, fails loudly without a GPU, raises the reference's
shape errors before any device work, and the host-side weight codecs match the
oracle bit for bit."""
import glob
import os
import re

import numpy as np
import pytest

from conftest import REPO


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        names |= set(re.findall(r"MRI_API\s+[\w\s\*]+?\b(mri_\w+)\s*\(", src))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "mri_matmul_int8" in names and "mri_matmul_q8_0_direct" in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol(mri):
    import ctypes
    lib = ctypes.CDLL(mri.library_path())
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_matches_header(mri):
    from importlib import import_module
    table = import_module("mini-rust-inference_b200._lib").SIGNATURES
    assert set(table) == declared_symbols()


def test_library_links_cudart_statically(mri):
    import subprocess
    out = subprocess.run(["ldd", mri.library_path()], capture_output=True, text=True).stdout
    assert "libcudart" not in out


def test_no_gpu_fails_loudly(mri):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(mri.CudaError):
        mri.Context(0)


class _WeightStub:
    """Only the attributes the products' shape checks read.  It has no handle
    and no context, so any device work would fail on it."""
    n_out, k_in = 3, 64


def test_shape_checks_run_before_device_work(mri):
    """The reference's error order (int8.rs:114-132, q8_direct.rs:230-246,
    q4_0.rs:101-119): a non-2-D input is InvalidShape and a K that differs
    from the weight's is ShapeMismatch, raised before anything touches the
    device (so here, without a GPU, no CudaError)."""
    w = _WeightStub()
    x3 = np.zeros((2, 3, 64), np.float32)
    x_bad_k = np.zeros((2, 32), np.float32)
    for fn in (mri.matmul_int8_from_f32, mri.matmul_q8_0_direct):
        with pytest.raises(mri.InvalidShape):
            fn(x3, w)
        with pytest.raises(mri.ShapeMismatch):
            fn(x_bad_k, w)
    with pytest.raises(mri.InvalidShape):
        mri.matmul_q4_0_dequant(x3, b"", 3, 64)
    with pytest.raises(mri.ShapeMismatch):
        mri.matmul_q4_0_dequant(x_bad_k, b"", 3, 64)
    assert issubclass(mri.InvalidShape, mri.TensorError) and issubclass(mri.ShapeMismatch, mri.TensorError)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_q8_0_codec_matches_oracle(mri, oracle, seed):
    rng = np.random.default_rng(seed)
    n, k = 7, 256
    w = rng.normal(0, 0.02 * (seed + 1), size=(n, k)).astype(np.float32)
    w[0, :32] = 0.0                       # all-zero block -> scale 0, quants 0
    w[1, 5] = np.float32(1e-6)            # tiny block scale (f16 subnormal branch)
    w[1, 32:64] = np.float32(3e-6)
    assert np.array_equal(mri.formats.quantize_q8_0(w, n, k), oracle.quantize_q8_0_matrix(w, n, k))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_q4_0_codec_matches_oracle(mri, oracle, seed):
    rng = np.random.default_rng(seed)
    n, k = 5, 128
    w = rng.normal(0, 0.5, size=(n, k)).astype(np.float32)
    w[2, :32] = 0.0                       # all-zero block -> 0x88 bytes
    assert np.array_equal(mri.formats.quantize_q4_0(w, n, k), oracle.quantize_q4_0_matrix(w, n, k))


def test_codecs_match_oracle_on_non_finite_values(mri, oracle):
    """create_q8_0_block / create_q4_0_block (dequant.rs:389-424, 706-749) on
    blocks holding inf, -inf, NaN, values past the f16 range and 1e30: the
    host codecs produce the oracle's bytes."""
    rng = np.random.default_rng(0)
    w = rng.normal(0, 1, size=(4, 64)).astype(np.float32)
    w[0, 3], w[1, 40], w[2, 7] = np.inf, -np.inf, np.nan
    w[3, :32], w[3, 33] = 1e30, 7e4
    with np.errstate(all="ignore"):
        assert np.array_equal(mri.formats.quantize_q8_0(w, 4, 64), oracle.quantize_q8_0_matrix(w, 4, 64))
        assert np.array_equal(mri.formats.quantize_q4_0(w, 4, 64), oracle.quantize_q4_0_matrix(w, 4, 64))


def test_f16_truncation_matches_oracle(mri, oracle):
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.normal(0, 1e-4, 2000), rng.normal(0, 100, 2000),
                           [0.0, -0.0, 65504.0, 70000.0, 1e-9, 6e-8, 6.1e-5, np.inf, -np.inf]]
                          ).astype(np.float32)
    got = mri.formats.f32_to_f16_trunc(vals)
    want = np.array([oracle.f32_to_f16(v) for v in vals], dtype=np.uint16)
    assert np.array_equal(got, want)


def test_dequantize_codecs_match_oracle(mri, oracle):
    rng = np.random.default_rng(4)
    w = rng.normal(0, 1, size=(3, 64)).astype(np.float32)
    b8 = oracle.quantize_q8_0_matrix(w, 3, 64)
    b4 = oracle.quantize_q4_0_matrix(w, 3, 64)
    assert np.array_equal(mri.formats.dequantize_q8_0(b8), oracle.dequantize_q8_0(b8))
    assert np.array_equal(mri.formats.dequantize_q4_0(b4), oracle.dequantize_q4_0(b4))


@pytest.mark.parametrize("m,k", [((4 << 20) // 1024 + 1, 1024), ((1 << 60) + 1, 16), (1, (4 << 20) + 16)])
def test_noalloc_size_check_precedes_device_work(mri, m, k):
    """The allocation-free entry point rejects an input larger than its fixed
    array before it touches the device (null pointers, no GPU here), also
    when m * k would wrap around in 64 bits."""
    lib = mri._lib.load()
    rc = lib.mri_matmul_int8_from_f32_noalloc(None, m, k, None, None, 8, None, None)
    assert rc == 6  # MRI_ERR_INVALID_ARGUMENT
    assert b"exceed the fixed scratch" in lib.mri_noalloc_last_error()


def test_option_constants_match_header(mri):
    """Every MRI_OPT_* value of include/mri_gpu.h has the same value as the
    Python mirror's OPT_* constant, and the option calls reject a null
    context without touching a device."""
    import ctypes
    header = open(os.path.join(REPO, "include", "mri_gpu.h")).read()
    found = dict(re.findall(r"MRI_OPT_(\w+)\s*=\s*(\d+)", header))
    assert len(found) >= 10
    for name, value in found.items():
        assert getattr(mri, "OPT_" + name) == int(value), name
    lib = mri._lib.load()
    assert lib.mri_ctx_set_option(None, 0, 1) == mri._lib.INVALID_ARGUMENT
    v = ctypes.c_int(-1)
    assert lib.mri_ctx_get_option(None, 0, ctypes.byref(v)) == mri._lib.INVALID_ARGUMENT
