"""GPU LlamaModelInt8 against the CPU model oracle (oracle/llama_oracle.py).

The projections are bit-exact INT8 products, but the glue (RMSNorm sums,
exp, attention order) is f32 in a different order, and a 1-ulp change in an
activation can move its INT8 code by one step.  Bar (the reference's own
model-level metric, forward_int8.rs:753-783, tightened from 10% to 2%):
max |logit error| / logit range < 0.02.
"""
import numpy as np
import pytest

import llama_oracle as lo

pytestmark = pytest.mark.gpu

TOL = 0.02


def rel_range_err(got, want):
    want = np.asarray(want, np.float32)
    rng = float(want.max() - want.min())
    return float(np.max(np.abs(np.asarray(got, np.float32) - want))) / max(rng, 1e-30)


def build_pair(mri, oracle, cfg, w):
    mcfg = mri.LlamaConfig(cfg["n_layers"], cfg["dim"], cfg["n_heads"], cfg["ffn_dim"], cfg["vocab"],
                           cfg["max_seq"], n_kv_heads=cfg["n_kv_heads"], rope_base=cfg["rope_base"],
                           rms_eps=cfg["rms_eps"])
    ref = lo.LlamaInt8Oracle(cfg, w)
    gpu = mri.LlamaModelInt8.from_weights(mcfg, w, rope=(ref.cos, ref.sin))
    return gpu, ref


def random_weights(cfg, seed):
    rng = np.random.default_rng(seed)
    d, V, ffn, hd = cfg["dim"], cfg["vocab"], cfg["ffn_dim"], cfg["dim"] // cfg["n_heads"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd

    def q(rows, cols):
        return (rng.integers(-127, 128, size=rows * cols, dtype=np.int8),
                rng.uniform(4e-4, 8e-4, size=rows).astype(np.float32) * np.float32(64.0 / np.sqrt(cols)))

    layers = [dict(wq=q(qd, d), wk=q(kvd, d), wv=q(kvd, d), wo=q(d, qd), wgate=q(ffn, d), wup=q(ffn, d),
                   wdown=q(d, ffn)) for _ in range(cfg["n_layers"])]
    return dict(token_embd=rng.uniform(-1, 1, size=V * d).astype(np.float32), layers=layers,
                attn_norm=rng.uniform(0.8, 1.2, size=cfg["n_layers"] * d).astype(np.float32),
                ffn_norm=rng.uniform(0.8, 1.2, size=cfg["n_layers"] * d).astype(np.float32),
                output_norm=np.ones(d, np.float32), output=q(V, d))


@pytest.fixture(scope="module")
def tiny(mri, oracle):
    cfg = lo.tiny_config()
    return build_pair(mri, oracle, cfg, lo.smooth_model_weights(cfg))


def test_forward_shapes_and_finite(tiny):
    gpu, _ = tiny
    assert gpu.forward([0]).shape == (1, 32)
    assert gpu.forward([0, 1, 2, 3]).shape == (4, 32)
    assert np.all(np.isfinite(gpu.forward([0, 5, 31])))


def test_forward_errors(mri, tiny):
    gpu, _ = tiny
    with pytest.raises(mri.InvalidShape):
        gpu.forward([])
    with pytest.raises(mri.InvalidShape):
        gpu.forward([32])


@pytest.mark.parametrize("toks", [[0], [0, 5, 15, 31], list(range(20))])
def test_forward_matches_oracle(tiny, toks):
    gpu, ref = tiny
    got, want = gpu.forward(toks), ref.forward(toks)
    for r in range(len(toks)):
        assert rel_range_err(got[r], want[r]) < TOL, r


def test_decode_matches_oracle(tiny):
    gpu, ref = tiny
    toks = [7, 3, 11, 2, 30, 9]
    gpu.forward(toks[:-1])
    ref.prefill_cached(toks[:-1])
    for step in range(3):
        pos = len(toks) - 1 + step
        tok = toks[-1] if step == 0 else (step * 5) % 32
        assert rel_range_err(gpu.forward_decode(tok, pos), ref.forward_decode(tok, pos)) < TOL
    assert gpu.kernels_per_decode_step() > 0


def _greedy_oracle(ref, prompt, n):
    logits = ref.prefill_cached(prompt)[-1]
    out, all_logits = [int(np.argmax(logits))], [logits]
    for i in range(n):
        logits = ref.forward_decode(out[-1], len(prompt) + i)
        all_logits.append(logits)
        out.append(int(np.argmax(logits)))
    return out, all_logits


def test_generate_greedy_matches_oracle(tiny):
    gpu, ref = tiny
    prompt = [1, 2, 3, 4, 5, 6, 7, 8]
    toks, pre_ms, dec_ms = gpu.generate_greedy(prompt, 10)
    want, logits = _greedy_oracle(ref, prompt, 10)
    assert len(toks) == 11 and pre_ms > 0 and dec_ms > 0
    for i, (g, w) in enumerate(zip(toks, want)):
        if g != w:
            # Only a near-tie may flip the greedy choice; after it the
            # sequences legitimately diverge.
            lg = logits[i]
            assert lg[w] - lg[g] <= TOL * (lg.max() - lg.min()), (i, g, w)
            break


def test_larger_gqa_model_uses_gemm_and_matches(mri, oracle):
    """dim 256, 4 query / 2 KV heads (GQA), 40-token prefill (tensor-core GEMM
    path for the projections) and decode (streaming GEMV path)."""
    cfg = dict(n_layers=2, dim=256, n_heads=4, n_kv_heads=2, ffn_dim=512, vocab=1000, max_seq=96,
               rope_base=10000.0, rms_eps=1e-5)
    gpu, ref = build_pair(mri, oracle, cfg, random_weights(cfg, 3))
    toks = list(np.random.default_rng(4).integers(0, 1000, size=40))
    got, want = gpu.forward(toks), ref.prefill_cached(toks)
    for r in (0, 17, 39):
        assert rel_range_err(got[r], want[r]) < TOL, r
    assert rel_range_err(gpu.forward_decode(5, 40), ref.forward_decode(5, 40)) < TOL


def test_head_dim_128_prefill_spans_tiles(mri, oracle):
    """Head dim 128 (the Llama-7B head), 4 query / 2 KV heads, a 150-token
    prefill: three 64-query blocks and three 64-key tiles of the tensor-core
    prefill attention, then a cached decode step."""
    cfg = dict(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, ffn_dim=768, vocab=500, max_seq=192,
               rope_base=10000.0, rms_eps=1e-5)
    gpu, ref = build_pair(mri, oracle, cfg, random_weights(cfg, 5))
    toks = list(np.random.default_rng(6).integers(0, 500, size=150))
    got, want = gpu.forward(toks), ref.prefill_cached(toks)
    for r in (0, 63, 64, 127, 128, 149):
        assert rel_range_err(got[r], want[r]) < TOL, r
    assert rel_range_err(gpu.forward_decode(7, 150), ref.forward_decode(7, 150)) < TOL


def test_prefill_split_key_walks(mri, oracle):
    """Head dim 64, a 330-token prefill: query blocks 1 and 2 walk 4 and 6
    key tiles, which two blocks split and the later one merges.  Rows on both
    sides of each split point against the oracle, and a second prefill gives
    the same logits bit for bit (the merge does not depend on which split
    finishes first)."""
    cfg = dict(n_layers=2, dim=256, n_heads=4, n_kv_heads=2, ffn_dim=512, vocab=300, max_seq=352,
               rope_base=10000.0, rms_eps=1e-5)
    gpu, ref = build_pair(mri, oracle, cfg, random_weights(cfg, 8))
    toks = list(np.random.default_rng(9).integers(0, 300, size=330))
    got, want = gpu.forward(toks), ref.prefill_cached(toks)
    for r in (0, 127, 128, 191, 192, 255, 256, 300, 329):
        assert rel_range_err(got[r], want[r]) < TOL, r
    np.testing.assert_array_equal(gpu.forward(toks), got)
    assert rel_range_err(gpu.forward_decode(11, 330), ref.forward_decode(11, 330)) < TOL


def test_decode_is_deterministic_at_scale(mri):
    """Two greedy runs and two decodes of the same step agree bit for bit on a
    model large enough that consecutive kernels overlap under programmatic
    dependent launch (a kernel that read a buffer through a stale cache line
    of its predecessor would make these differ)."""
    cfg = mri.LlamaConfig(4, 2048, 16, 5632, 8000, 160)
    m = mri.LlamaModelInt8.random(cfg, seed=3)
    prompt = np.random.default_rng(1).integers(0, 8000, size=96).astype(np.uint32)
    a, _, _ = m.generate_greedy(prompt, 24)
    b, _, _ = m.generate_greedy(prompt, 24)
    np.testing.assert_array_equal(a, b)
    m.forward(prompt)
    la = m.forward_decode(int(a[0]), 96)
    lb = m.forward_decode(int(a[0]), 96)
    np.testing.assert_array_equal(la, lb)


# ── model-level bars calibrated on a second correct restatement ─────────────
#
# The model quantizes every projection input per tensor to INT8, so its output
# is a discontinuous function of the f32 glue: a 1-ulp difference in an RMSNorm
# sum or an attention weight moves some INT8 codes by one step.  Two correct f32
# implementations that differ only in rounding order therefore drift apart by
# an amount set by the model's size, not by any error: the oracle with its glue
# accumulated in float64 (llama_oracle glue="f64") differs from the oracle
# itself by a median of ~1.9% of the block output's range per row at the 7B
# dimensions (one block) and ~4.5% of the logit range (two blocks and the head),
# more than the 2% bar used on the small configurations above.  The tests below
# therefore hold the GPU's per-row errors against that drift, measured in the
# test on the same inputs: its median, 90th percentile and maximum may exceed
# the f64 restatement's by a small factor.  A semantic error (a wrong position,
# cache row or mask, or the per-chunk activation scale of a chunked prefill
# compared with one prefill) lands far outside: each test also checks that the
# bar would reject such a difference.

def row_errors(got, want, base=None):
    """Per row: max |got - want| / range of want (of want - base with `base`,
    i.e. of a block's own contribution to its residual input)."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    out = []
    for r in range(want.shape[0]):
        ref = want[r] if base is None else want[r] - np.asarray(base[r], np.float32)
        rng = float(ref.max() - ref.min())
        out.append(float(np.max(np.abs(got[r] - want[r]))) / max(rng, 1e-30))
    return np.array(out)


def noise_bar(e_alt, slack=0.003):
    """Bounds on (median, p90, max) of a row-error distribution: those of the
    f64 restatement's errors, 1.25x (1.5x for the max) plus `slack`."""
    return (1.25 * np.median(e_alt) + slack, 1.25 * np.quantile(e_alt, 0.9) + slack,
            1.5 * e_alt.max() + 2 * slack)


def within(e, bar):
    return np.median(e) <= bar[0] and np.quantile(e, 0.9) <= bar[1] and e.max() <= bar[2]


def describe(e, bar):
    return (f"median {np.median(e):.4f} (bar {bar[0]:.4f}), p90 {np.quantile(e, 0.9):.4f} (bar {bar[1]:.4f}), "
            f"max {e.max():.4f} (bar {bar[2]:.4f})")


SEVEN_B = dict(n_layers=2, dim=4096, n_heads=32, n_kv_heads=32, ffn_dim=11008, vocab=32000, max_seq=520,
               rope_base=10000.0, rms_eps=1e-5)


@pytest.fixture(scope="module")
def seven_b(mri, oracle):
    """Two layers of the benchmarked Llama-7B shape (d 4096, 32 heads of 128,
    FFN 11008, vocab 32000) with the oracle and the f64-glue restatement."""
    w = random_weights(SEVEN_B, 12)
    gpu, ref = build_pair(mri, oracle, SEVEN_B, w)
    return gpu, ref, w


def test_7b_dims_blocks_match_oracle(mri, oracle, seven_b):
    """TransformerBlockInt8::forward_cached_parallel at the 7B dimensions
    through the block entry point: both layers on the same 512-row input (the
    benchmarked prefill: tensor-core GEMMs, tensor-core attention with split
    key walks), the same rows in two chunks at an offset that cuts a query
    block, and one row at position 512 (streaming GEMVs, the prefill attention
    over the whole cache).  Every row against the oracle, within the f64
    restatement's drift; the bar rejects the chunked-versus-whole difference
    of the reference's own per-chunk quantization."""
    gpu, _, w = seven_b
    n, cut = 512, 259
    x = np.random.default_rng(5).uniform(-1, 1, size=(n, SEVEN_B["dim"])).astype(np.float32)
    for layer in (0, 1):
        ref, alt = lo.LlamaInt8Oracle(SEVEN_B, w), lo.LlamaInt8Oracle(SEVEN_B, w, glue="f64")
        a, b, g = ref.block_forward(layer, x, 0), alt.block_forward(layer, x, 0), gpu.block_forward(layer, x, 0)
        bar = noise_bar(row_errors(b, a, x))
        e = row_errors(g, a, x)
        assert within(e, bar), (layer, "whole", describe(e, bar))
        a2 = np.concatenate([ref.block_forward(layer, x[:cut], 0), ref.block_forward(layer, x[cut:], cut)])
        b2 = np.concatenate([alt.block_forward(layer, x[:cut], 0), alt.block_forward(layer, x[cut:], cut)])
        g2 = np.concatenate([gpu.block_forward(layer, x[:cut], 0), gpu.block_forward(layer, x[cut:], cut)])
        bar2 = noise_bar(row_errors(b2, a2, x))
        e2 = row_errors(g2, a2, x)
        assert within(e2, bar2), (layer, "chunks", describe(e2, bar2))
        assert not within(row_errors(a2, a, x), bar), "the bar must separate chunked from whole prefill"
        a3, b3, g3 = (ref.block_forward(layer, x[:1], n), alt.block_forward(layer, x[:1], n),
                      gpu.block_forward(layer, x[:1], n))
        e3, f3 = row_errors(g3, a3, x[:1]), row_errors(b3, a3, x[:1])
        assert e3[0] <= 1.5 * f3[0] + 0.006, (layer, "one row", e3[0], f3[0])
    assert gpu.attention_fallbacks() == 0


def test_7b_dims_model_matches_oracle(mri, oracle, seven_b):
    """The whole two-layer 7B-shaped model: the 512-token prefill of
    BASELINE's model config and 8 greedy decode steps through the captured
    decode graph (streaming GEMVs with the RoPE/KV-cache and SwiGLU
    epilogues, split decode attention), logits against the oracle within the
    f64 restatement's drift."""
    gpu, _, w = seven_b
    toks = list(np.random.default_rng(13).integers(0, 32000, size=512))
    ref, alt = lo.LlamaInt8Oracle(SEVEN_B, w), lo.LlamaInt8Oracle(SEVEN_B, w, glue="f64")
    a, b, g = ref.prefill_cached(toks), alt.prefill_cached(toks), gpu.forward(toks)
    bar = noise_bar(row_errors(b, a), slack=0.005)
    e = row_errors(g, a)
    assert within(e, bar), describe(e, bar)
    tok = int(np.argmax(a[-1]))
    da, db, dg = [], [], []
    for step in range(8):
        pos = 512 + step
        da.append(ref.forward_decode(tok, pos))
        db.append(alt.forward_decode(tok, pos))
        dg.append(gpu.forward_decode(tok, pos))
        tok = int(np.argmax(da[-1]))
    bar = noise_bar(row_errors(db, da), slack=0.005)
    e = row_errors(dg, da)
    assert within(e, bar), describe(e, bar)
    assert gpu.attention_fallbacks() == 0


def _offset_cfg():
    return dict(n_layers=2, dim=256, n_heads=4, n_kv_heads=2, ffn_dim=512, vocab=300, max_seq=400,
                rope_base=10000.0, rms_eps=1e-5)


def test_forward_at_chunks_match_oracle_chunks(mri, oracle):
    """forward_cached_parallel's block loop at start_pos > 0 through the whole
    model (forward_int8.rs:232-249): a 350-token prompt prefilled in chunks of
    170 (GEMM), 5 (streaming GEMV) and 175 tokens (GEMM; key walks split over
    two blocks), at offsets that cut through query blocks and key tiles,
    against the oracle prefilling the same chunks (each chunk's activations
    are quantized with their own per-tensor scale, as in the reference, so a
    chunked prefill is not one prefill).  Then a decode step continues from
    the chunked cache, and a chunk repeated on the same cache is
    bit-identical."""
    cfg = _offset_cfg()
    w = random_weights(cfg, 31)
    gpu, ref = build_pair(mri, oracle, cfg, w)
    alt = lo.LlamaInt8Oracle(cfg, w, glue="f64")
    toks = list(np.random.default_rng(32).integers(0, 300, size=350))
    cuts = [(0, 170), (170, 175), (175, 350)]
    g = np.concatenate([gpu.forward_at(toks[s:e], s) for s, e in cuts])
    a = np.concatenate([ref.forward_cached(toks[s:e], s) for s, e in cuts])
    b = np.concatenate([alt.forward_cached(toks[s:e], s) for s, e in cuts])
    bar = noise_bar(row_errors(b, a), slack=0.005)
    e = row_errors(g, a)
    assert within(e, bar), describe(e, bar)
    whole = lo.LlamaInt8Oracle(cfg, w).prefill_cached(toks)
    assert not within(row_errors(a, whole), bar), "the bar must separate chunked from whole prefill"
    d_g, d_a, d_b = gpu.forward_decode(7, 350), ref.forward_decode(7, 350), alt.forward_decode(7, 350)
    assert row_errors([d_g], [d_a])[0] <= 1.5 * row_errors([d_b], [d_a])[0] + 0.01
    np.testing.assert_array_equal(gpu.forward_at(toks[175:], 175), g[175:])


def test_forward_at_rejects_positions_past_max_seq(mri, oracle):
    cfg = _offset_cfg()
    gpu, _ = build_pair(mri, oracle, cfg, random_weights(cfg, 33))
    with pytest.raises(mri.InvalidShape):
        gpu.forward_at([1, 2, 3], 398)
    with pytest.raises(mri.InvalidShape):
        gpu.forward_at([], 0)
    with pytest.raises(mri.InvalidShape):
        gpu.block_forward(2, np.zeros((1, 256), np.float32), 0)


@pytest.mark.parametrize("option,value", [("OPT_TC_ATTN", 0), ("OPT_FA_SPLIT", 0)])
def test_prefill_attention_variants_match_oracle(mri, oracle, option, value):
    """The CUDA-core prefill attention (OPT_TC_ATTN = 0) and the tensor-core
    kernel without split key walks (OPT_FA_SPLIT = 0) on the 330-token
    head-dim-64 case: every row against the oracle within the f64
    restatement's drift."""
    cfg = dict(n_layers=2, dim=256, n_heads=4, n_kv_heads=2, ffn_dim=512, vocab=300, max_seq=352,
               rope_base=10000.0, rms_eps=1e-5)
    w = random_weights(cfg, 8)
    gpu, ref = build_pair(mri, oracle, cfg, w)
    gpu.set_option(getattr(mri, option), value)
    toks = list(np.random.default_rng(9).integers(0, 300, size=330))
    a, b, g = ref.prefill_cached(toks), lo.LlamaInt8Oracle(cfg, w, glue="f64").prefill_cached(toks), gpu.forward(toks)
    bar = noise_bar(row_errors(b, a), slack=0.005)
    e = row_errors(g, a)
    assert within(e, bar), describe(e, bar)


def test_prefill_attention_beyond_f16_range_falls_back(mri, oracle):
    """Layer 0's q rows scaled so that q lies far beyond the f16 range
    (|q| > 65504), which the tensor-core prefill attention cannot represent:
    the call is run again on the f32 CUDA-core attention, its logits are
    bit-identical to a forward with that kernel selected outright, and they
    match the oracle within the f64 restatement's drift."""
    cfg = dict(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, ffn_dim=768, vocab=500, max_seq=192,
               rope_base=10000.0, rms_eps=1e-5)
    w = random_weights(cfg, 41)
    wq, sq = w["layers"][0]["wq"]
    w["layers"][0]["wq"] = (wq, (sq * np.float32(1e5)).astype(np.float32))
    gpu, ref = build_pair(mri, oracle, cfg, w)
    toks = list(np.random.default_rng(42).integers(0, 500, size=150))
    got = gpu.forward(toks)
    assert gpu.attention_fallbacks() == 1
    a, b = ref.prefill_cached(toks), lo.LlamaInt8Oracle(cfg, w, glue="f64").prefill_cached(toks)
    bar = noise_bar(row_errors(b, a), slack=0.005)
    e = row_errors(got, a)
    assert within(e, bar), describe(e, bar)
    gpu.set_option(mri.OPT_TC_ATTN, 0)
    np.testing.assert_array_equal(gpu.forward(toks), got)
    assert gpu.attention_fallbacks() == 1
