"""The LlamaModelInt8 oracle against the reference's model-level tests
(model/llama/forward_int8.rs:653-741) and its own cache consistency."""
import numpy as np
import pytest

import llama_oracle as lo


@pytest.fixture(scope="module")
def model(oracle):
    cfg = lo.tiny_config()
    return lo.LlamaInt8Oracle(cfg, lo.smooth_model_weights(cfg))


def test_forward_shapes(model):
    # forward_int8.rs:653-671
    assert model.forward([0]).shape == (1, 32)
    assert model.forward([0, 1, 2, 3]).shape == (4, 32)


def test_forward_no_nan_or_inf(model):
    # forward_int8.rs:675-684
    assert np.all(np.isfinite(model.forward([0, 5, 31])))


def test_forward_errors(model):
    # forward_int8.rs:688-699
    with pytest.raises(ValueError):
        model.forward([])
    with pytest.raises(ValueError):
        model.forward([32])


def test_decode_length_and_finite(model):
    # forward_int8.rs:716-741
    assert model.forward_decode(0, 0).shape == (32,)
    assert np.all(np.isfinite(model.forward_decode(5, 0)))


def test_cached_prefill_equals_forward(model):
    """Writing the cache does not change the prefill arithmetic."""
    toks = [3, 1, 4, 1, 5, 9, 2, 6]
    assert np.array_equal(model.forward(toks), model.prefill_cached(toks))


def test_decode_after_prefill_matches_longer_forward(model):
    """forward_decode(t_n, n) after caching t_0..t_{n-1} sees the same context
    as forward(t_0..t_n): logits agree closely (the per-tensor activation
    scale differs: one row vs n+1 rows)."""
    toks = [7, 3, 11, 2, 30]
    model.prefill_cached(toks[:-1])
    dec = model.forward_decode(toks[-1], len(toks) - 1)
    full = model.forward(toks)[-1]
    rng = full.max() - full.min()
    assert np.max(np.abs(dec - full)) / rng < 0.1
