"""GGUF loading: the container reader (CPU) and the device loader (GPU).

CPU tests restate the reference's own header / metadata / tensor-table /
LlamaConfig tests (src/gguf/header.rs:318-420, src/gguf/metadata.rs tests,
src/gguf/tensor_info.rs tests, src/model/llama/config.rs:160-300) against the
Python reader, and check the oracle's extract() against the codecs.

GPU tests: the device loader (dequantize + per-channel requantize of
from_loader, forward_int8.rs:461-507) must give the oracle's
quantize_tensor(extract()) bit for bit, and a model loaded from a GGUF file
must give the same logits as the same weights loaded through
LlamaModelInt8::new (from_weights).
"""
import struct

import numpy as np
import pytest

from conftest import load_mri

gguf = __import__("importlib").import_module("mini-rust-inference_b200.gguf")


def header_bytes(magic=b"GGUF", version=3, n_tensors=0, n_kv=0):
    return magic + struct.pack("<IQQ", version, n_tensors, n_kv)


# ── header (header.rs:322-395) ───────────────────────────────────────────────

def test_valid_header_v3():
    assert gguf.read_header(header_bytes(version=3, n_tensors=10, n_kv=5)) == (3, 10, 5)


def test_valid_header_v2():
    assert gguf.read_header(header_bytes(version=2, n_tensors=100, n_kv=20)) == (2, 100, 20)


def test_invalid_magic():
    with pytest.raises(gguf.InvalidMagic):
        gguf.read_header(header_bytes(magic=b"GGML"))


@pytest.mark.parametrize("version", [1, 4])
def test_unsupported_version(version):
    with pytest.raises(gguf.UnsupportedVersion):
        gguf.read_header(header_bytes(version=version))


@pytest.mark.parametrize("data", [b"GGUF", b""])
def test_truncated_or_empty_header(data):
    with pytest.raises(gguf.UnexpectedEof):
        gguf.read_header(data)


# ── metadata and tensor table ───────────────────────────────────────────────

ALL_VALUES = {
    "u8": (gguf.UINT8, 200), "i8": (gguf.INT8, -100), "u16": (gguf.UINT16, 60000),
    "i16": (gguf.INT16, -30000), "u32": (gguf.UINT32, 4_000_000_000), "i32": (gguf.INT32, -2_000_000_000),
    "f32": (gguf.FLOAT32, 0.5), "bool": (gguf.BOOL, True), "str": (gguf.STRING, "llama"),
    "u64": (gguf.UINT64, 1 << 40), "i64": (gguf.INT64, -(1 << 40)), "f64": (gguf.FLOAT64, 0.1),
    "arr_u32": (gguf.ARRAY, (gguf.UINT32, [1, 2, 3])),
    "arr_str": (gguf.ARRAY, (gguf.STRING, ["a", "bc", ""])),
}


def test_metadata_roundtrip_every_type(tmp_path):
    p = tmp_path / "m.gguf"
    gguf.write_gguf(p, ALL_VALUES, [])
    g = gguf.GgufFile(p)
    assert g.version == 3 and len(g.metadata) == len(ALL_VALUES)
    for k, v in ALL_VALUES.items():
        assert g.metadata.get(k) == v, k
    assert g.metadata.get_u32("u8") == 200 and g.metadata.get_u32("u64") is None
    assert g.metadata.get_u64("u64") == 1 << 40 and g.metadata.get_f32("f64") is None
    assert g.metadata.get_string_array("arr_str") == ["a", "bc", ""]


def _kv(key, vtype, payload):
    return struct.pack("<Q", len(key)) + key + struct.pack("<I", vtype) + payload


def test_duplicate_key_rejected():
    one = _kv(b"k", gguf.UINT32, struct.pack("<I", 1))
    with pytest.raises(gguf.DuplicateKey):
        gguf.GgufFile.from_bytes(header_bytes(n_kv=2) + one + one)


def test_nested_array_rejected():
    inner = struct.pack("<IQ", gguf.ARRAY, 1) + struct.pack("<IQ", gguf.UINT8, 0)
    with pytest.raises(gguf.NestedArray):
        gguf.GgufFile.from_bytes(header_bytes(n_kv=1) + _kv(b"a", gguf.ARRAY, inner))


def test_invalid_bool_and_unknown_type():
    with pytest.raises(gguf.InvalidBool):
        gguf.GgufFile.from_bytes(header_bytes(n_kv=1) + _kv(b"b", gguf.BOOL, b"\x02"))
    with pytest.raises(gguf.UnknownValueType):
        gguf.GgufFile.from_bytes(header_bytes(n_kv=1) + _kv(b"x", 13, b""))


def test_truncated_metadata():
    with pytest.raises(gguf.UnexpectedEof):
        gguf.GgufFile.from_bytes(header_bytes(n_kv=1) + struct.pack("<Q", 10) + b"abc")


def test_tensor_table_dims_offsets_and_alignment(tmp_path):
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    b = np.arange(5, dtype=np.float32)
    for align in (None, 64):
        meta = {} if align is None else {"general.alignment": (gguf.UINT32, align)}
        p = tmp_path / f"t{align}.gguf"
        gguf.write_gguf(p, meta, [("a", a.shape, gguf.F32, a.tobytes()), ("b", b.shape, gguf.F32, b.tobytes())],
                        alignment=align or gguf.DEFAULT_ALIGNMENT)
        g = gguf.GgufFile(p)
        assert g.alignment == (align or 32) and g.data_offset % g.alignment == 0
        ia, ib = g.tensor("a"), g.tensor("b")
        assert ia.dims == (3, 2) and ia.shape_row_major() == (2, 3) and ia.size_bytes() == 24
        assert ib.offset % g.alignment == 0
        np.testing.assert_array_equal(g.tensor_data("a").view(np.float32), a.ravel())
        np.testing.assert_array_equal(g.tensor_data("b").view(np.float32), b)
        with pytest.raises(gguf.KeyNotFound):
            g.tensor("missing")
        g.close()


def test_tensor_table_errors():
    def info(name, n_dims, dtype=0):
        return (struct.pack("<Q", len(name)) + name + struct.pack("<I", n_dims) + struct.pack("<Q", 1) * n_dims
                + struct.pack("<IQ", dtype, 0))
    with pytest.raises(gguf.ValueOutOfRange):
        gguf.GgufFile.from_bytes(header_bytes(n_tensors=1) + info(b"t", 9))
    with pytest.raises(gguf.KeyNotFound):
        gguf.GgufFile.from_bytes(header_bytes(n_tensors=2) + info(b"t", 1) + info(b"t", 1))
    with pytest.raises(gguf.UnknownValueType):  # ggml type 4 does not exist
        gguf.GgufFile.from_bytes(header_bytes(n_tensors=1) + info(b"t", 1, dtype=4))


def test_tensor_data_outside_file_is_unavailable():
    t = struct.pack("<Q", 1) + b"t" + struct.pack("<IQ", 1, 1000) + struct.pack("<IQ", 0, 0)
    g = gguf.GgufFile.from_bytes(header_bytes(n_tensors=1) + t)
    assert g.tensor_data("t") is None


# ── LlamaConfig::from_metadata (config.rs:160-300) ──────────────────────────

def minimal_meta(**extra):
    e = {"llama.block_count": (gguf.UINT32, 32), "llama.embedding_length": (gguf.UINT32, 4096),
         "llama.attention.head_count": (gguf.UINT32, 32), "llama.feed_forward_length": (gguf.UINT32, 11008),
         "llama.context_length": (gguf.UINT32, 4096), "llama.vocab_size": (gguf.UINT32, 32000)}
    e.update(extra)
    return gguf.Metadata({k: v for k, v in e.items() if v is not None})


def test_config_from_minimal_metadata():
    c = gguf.llama_config(minimal_meta())
    assert (c["block_count"], c["embedding_length"], c["n_heads"], c["n_kv_heads"]) == (32, 4096, 32, 32)
    assert (c["feed_forward_length"], c["context_length"], c["vocab_size"]) == (11008, 4096, 32000)
    assert c["rope_freq_base"] == 10000.0 and abs(c["rms_norm_eps"] - 1e-5) < 1e-10
    assert c["embedding_length"] // c["n_heads"] == 128


def test_config_optional_fields():
    c = gguf.llama_config(minimal_meta(**{"llama.attention.head_count_kv": (gguf.UINT32, 8),
                                          "llama.rope.freq_base": (gguf.FLOAT32, 500000.0),
                                          "llama.attention.layer_norm_rms_epsilon": (gguf.FLOAT32, 1e-6)}))
    assert c["n_kv_heads"] == 8 and c["rope_freq_base"] == 500000.0 and c["rms_norm_eps"] == 1e-6


def test_config_vocab_from_token_list_and_u64():
    toks = (gguf.STRING, [f"tok{i}" for i in range(500)])
    c = gguf.llama_config(minimal_meta(**{"llama.vocab_size": None, "tokenizer.ggml.tokens": (gguf.ARRAY, toks)}))
    assert c["vocab_size"] == 500
    c = gguf.llama_config(minimal_meta(**{"llama.vocab_size": (gguf.UINT64, 32000)}))
    assert c["vocab_size"] == 32000


def test_config_errors():
    with pytest.raises(gguf.MissingMetadataKey):
        gguf.llama_config(gguf.Metadata())
    with pytest.raises(gguf.InvalidConfig):
        gguf.llama_config(minimal_meta(**{"llama.attention.head_count": (gguf.UINT32, 7)}))
    with pytest.raises(gguf.InvalidConfig):
        gguf.llama_config(minimal_meta(**{"llama.attention.head_count_kv": (gguf.UINT32, 5)}))


# ── oracle extract() against the codecs ─────────────────────────────────────

def encode(oracle, w, n, k, ggml_type):
    """f32 [n, k] -> the raw GGUF bytes of that tensor stored as ggml_type."""
    w = np.ascontiguousarray(w, np.float32).reshape(n, k)
    if ggml_type == gguf.F32:
        return w.tobytes()
    if ggml_type == gguf.F16:
        return np.array([oracle.f32_to_f16(float(v)) for v in w.ravel()], np.uint16).tobytes()
    if ggml_type == gguf.Q8_0:
        return oracle.quantize_q8_0_matrix(w, n, k).tobytes()
    return oracle.quantize_q4_0_matrix(w, n, k).tobytes()


@pytest.mark.parametrize("ggml_type", [gguf.F32, gguf.F16, gguf.Q8_0, gguf.Q4_0])
def test_oracle_extract_matches_codecs(oracle, ggml_type):
    rng = np.random.default_rng(5)
    w = rng.normal(0, 0.05, size=(4, 64)).astype(np.float32)
    raw = encode(oracle, w, 4, 64, ggml_type)
    got = oracle.extract(ggml_type, np.frombuffer(raw, np.uint8))
    if ggml_type == gguf.F32:
        np.testing.assert_array_equal(got, w.ravel())
    elif ggml_type == gguf.F16:
        # IEEE half decode of the stored bits (numpy's is exact too).
        np.testing.assert_array_equal(got, np.frombuffer(raw, np.float16).astype(np.float32))
    else:
        # Within half a quantization step of the block scale.
        step = np.abs(w).max() / (127 if ggml_type == gguf.Q8_0 else 7)
        assert np.max(np.abs(got - w.ravel())) <= 0.51 * step
    data, scales = oracle.quantize_tensor(ggml_type, np.frombuffer(raw, np.uint8), 4, 64)
    d2, s2 = oracle.quantize_per_channel(got, 4, 64)
    np.testing.assert_array_equal(data, d2)
    np.testing.assert_array_equal(scales, s2)


# ── device loader (GPU) ─────────────────────────────────────────────────────

LOAD_SHAPES = [(1, 32), (7, 96), (300, 4096), (33, 11008)]


@pytest.mark.gpu
@pytest.mark.parametrize("ggml_type", [gguf.F32, gguf.F16, gguf.Q8_0, gguf.Q4_0])
@pytest.mark.parametrize("n,k", LOAD_SHAPES)
def test_qmatrix_from_gguf_bit_exact(mri, gpu_ctx, oracle, ggml_type, n, k):
    rng = np.random.default_rng(n * 7 + k)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    w[0, :5] = [0.0, -0.0, 1e-30, -3.5, 2.25]  # zeros, a subnormal-scale value, exact halves
    if n > 2:
        w[2] = 0.0  # an all-zero row: scale 1.0
    if ggml_type == gguf.F16:
        raw = w.astype(np.float16).tobytes()  # any half bit patterns will do as input
    else:
        raw = encode(oracle, w, n, k, ggml_type)
    raw = np.frombuffer(raw, np.uint8)
    qm = mri.QuantizedMatrix.from_gguf(ggml_type, raw, n, k, ctx=gpu_ctx)
    want_d, want_s = oracle.quantize_tensor(ggml_type, raw, n, k)
    np.testing.assert_array_equal(qm.scales, want_s)
    np.testing.assert_array_equal(qm.data, want_d)


@pytest.mark.gpu
@pytest.mark.parametrize("ggml_type", [gguf.F16, gguf.Q8_0, gguf.Q4_0])
def test_gguf_dequant_bit_exact(mri, gpu_ctx, oracle, ggml_type):
    rng = np.random.default_rng(11)
    w = rng.normal(0, 1.0, size=(3, 160)).astype(np.float32)
    raw = np.frombuffer(encode(oracle, w, 3, 160, ggml_type), np.uint8)
    got = mri.gguf_dequant(ggml_type, raw, w.size, ctx=gpu_ctx)
    np.testing.assert_array_equal(got, oracle.extract(ggml_type, raw))


@pytest.mark.gpu
def test_gguf_dequant_into_device_tensor(mri, gpu_ctx, oracle):
    """The `out=` form fills a caller's CUDA tensor, after the fill that
    torch queued on it."""
    import torch
    rng = np.random.default_rng(12)
    w = rng.normal(0, 1.0, size=(3, 160)).astype(np.float32)
    raw = np.frombuffer(encode(oracle, w, 3, 160, gguf.Q8_0), np.uint8)
    out = torch.full((w.size,), float("nan"), device="cuda")
    got = mri.gguf_dequant(gguf.Q8_0, raw, w.size, out=out, ctx=gpu_ctx)
    assert got is out
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.extract(gguf.Q8_0, raw))


@pytest.mark.gpu
def test_block_rows_not_on_block_boundary(mri, gpu_ctx, oracle):
    """[2, 48] Q8_0: 96 values = 3 blocks, the middle one straddles the rows
    (extract dequantizes the flat block stream)."""
    rng = np.random.default_rng(3)
    flat = rng.normal(0, 0.1, size=96).astype(np.float32)
    raw = np.frombuffer(oracle.quantize_q8_0_matrix(flat, 1, 96).tobytes(), np.uint8)
    qm = mri.QuantizedMatrix.from_gguf(gguf.Q8_0, raw, 2, 48, ctx=gpu_ctx)
    want_d, want_s = oracle.quantize_tensor(gguf.Q8_0, raw, 2, 48)
    np.testing.assert_array_equal(qm.data, want_d)
    np.testing.assert_array_equal(qm.scales, want_s)


@pytest.mark.gpu
def test_from_gguf_errors(mri, gpu_ctx):
    raw = np.zeros(34, np.uint8)
    with pytest.raises(ValueError):  # TypeMismatch: Q4_1
        mri.QuantizedMatrix.from_gguf(3, np.zeros(20, np.uint8), 1, 32, ctx=gpu_ctx)
    with pytest.raises(mri.ShapeMismatch):  # 31 values of Q8_0
        mri.QuantizedMatrix.from_gguf(gguf.Q8_0, raw, 1, 31, ctx=gpu_ctx)
    with pytest.raises(mri.ShapeMismatch):  # one byte short
        mri.QuantizedMatrix.from_gguf(gguf.Q8_0, raw[:33], 1, 32, ctx=gpu_ctx)
    with pytest.raises(mri.ShapeMismatch):
        mri.QuantizedMatrix.from_gguf(gguf.F32, np.zeros(12, np.uint8), 1, 4, ctx=gpu_ctx)


TINY = dict(n_layers=2, dim=128, n_heads=4, n_kv_heads=2, ffn_dim=352, vocab=96, max_seq=64,
            rope_base=10000.0, rms_eps=1e-5)

# Storage type of each tensor in the synthetic file: every supported type on
# some projection, the embedding in F16, norms in F32.
TYPES = {"token_embd.weight": gguf.F16, "output_norm.weight": gguf.F32, "output.weight": gguf.Q8_0,
         "attn_q.weight": gguf.Q8_0, "attn_k.weight": gguf.Q4_0, "attn_v.weight": gguf.F16,
         "attn_output.weight": gguf.F32, "attn_norm.weight": gguf.F32, "ffn_gate.weight": gguf.Q4_0,
         "ffn_up.weight": gguf.Q8_0, "ffn_down.weight": gguf.F16, "ffn_norm.weight": gguf.F32}


def write_tiny_model(path, oracle, seed=0):
    """Writes a GGUF llama file of f32 weights stored in mixed types; returns
    the from_weights dict of what from_loader makes of it (oracle side)."""
    c = TINY
    rng = np.random.default_rng(seed)
    d, hd = c["dim"], c["dim"] // c["n_heads"]
    qd, kvd, F, V = c["n_heads"] * hd, c["n_kv_heads"] * hd, c["ffn_dim"], c["vocab"]
    shapes = {"attn_q.weight": (qd, d), "attn_k.weight": (kvd, d), "attn_v.weight": (kvd, d),
              "attn_output.weight": (d, qd), "ffn_gate.weight": (F, d), "ffn_up.weight": (F, d),
              "ffn_down.weight": (d, F)}
    tensors, w = [], {"layers": [dict() for _ in range(c["n_layers"])]}

    def add(name, key, shape, values, quantize):
        t = TYPES[key]
        n, k = (1, shape[0]) if len(shape) == 1 else shape
        raw = encode(oracle, values, n, k, t)
        tensors.append((name, shape, t, raw))
        u8 = np.frombuffer(raw, np.uint8)
        return oracle.quantize_tensor(t, u8, n, k) if quantize else oracle.extract(t, u8)

    w["token_embd"] = add("token_embd.weight", "token_embd.weight", (V, d),
                          rng.normal(0, 1.0, (V, d)).astype(np.float32), False)
    w["output_norm"] = add("output_norm.weight", "output_norm.weight", (d,),
                           rng.uniform(0.8, 1.2, d).astype(np.float32), False)
    w["output"] = add("output.weight", "output.weight", (V, d), rng.normal(0, 0.05, (V, d)).astype(np.float32),
                      True)
    an, fn = [], []
    for li in range(c["n_layers"]):
        for key, shape in shapes.items():
            vals = rng.normal(0, 0.3 / np.sqrt(shape[1]), shape).astype(np.float32)
            w["layers"][li][{"attn_q.weight": "wq", "attn_k.weight": "wk", "attn_v.weight": "wv",
                             "attn_output.weight": "wo", "ffn_gate.weight": "wgate", "ffn_up.weight": "wup",
                             "ffn_down.weight": "wdown"}[key]] = add(gguf.weight_name(li, key), key, shape, vals,
                                                                      True)
        an.append(add(gguf.weight_name(li, "attn_norm.weight"), "attn_norm.weight", (d,),
                      rng.uniform(0.8, 1.2, d).astype(np.float32), False))
        fn.append(add(gguf.weight_name(li, "ffn_norm.weight"), "ffn_norm.weight", (d,),
                      rng.uniform(0.8, 1.2, d).astype(np.float32), False))
    w["attn_norm"], w["ffn_norm"] = np.concatenate(an), np.concatenate(fn)
    meta = {"general.architecture": (gguf.STRING, "llama"),
            "llama.block_count": (gguf.UINT32, c["n_layers"]), "llama.embedding_length": (gguf.UINT32, d),
            "llama.attention.head_count": (gguf.UINT32, c["n_heads"]),
            "llama.attention.head_count_kv": (gguf.UINT32, c["n_kv_heads"]),
            "llama.feed_forward_length": (gguf.UINT32, F), "llama.context_length": (gguf.UINT32, c["max_seq"]),
            "llama.vocab_size": (gguf.UINT32, V), "llama.rope.freq_base": (gguf.FLOAT32, c["rope_base"]),
            "llama.attention.layer_norm_rms_epsilon": (gguf.FLOAT32, c["rms_eps"])}
    gguf.write_gguf(path, meta, tensors)
    return w


def test_tiny_model_file_parses(tmp_path, oracle):
    p = tmp_path / "tiny.gguf"
    write_tiny_model(p, oracle)
    g = gguf.GgufFile(p)
    c = gguf.llama_config(g.metadata)
    assert (c["block_count"], c["embedding_length"], c["n_kv_heads"], c["vocab_size"]) == (2, 128, 2, 96)
    assert len(g.tensors) == 3 + 9 * TINY["n_layers"]
    assert g.tensor("blk.1.ffn_down.weight").shape_row_major() == (128, 352)
    assert g.tensor("blk.0.attn_norm.weight").shape_row_major() == (128,)
    for name in g.tensors:
        assert g.tensor_data(name) is not None


@pytest.mark.gpu
def test_model_from_gguf_equals_from_weights(mri, gpu_ctx, oracle, tmp_path):
    p = tmp_path / "tiny.gguf"
    w = write_tiny_model(p, oracle, seed=1)
    c = TINY
    cfg = mri.LlamaConfig(c["n_layers"], c["dim"], c["n_heads"], c["ffn_dim"], c["vocab"], c["max_seq"],
                          n_kv_heads=c["n_kv_heads"], rope_base=c["rope_base"], rms_eps=c["rms_eps"])
    ref = mri.LlamaModelInt8.from_weights(cfg, w, ctx=gpu_ctx)
    got = mri.LlamaModelInt8.from_gguf(p, ctx=gpu_ctx)
    assert got.cfg.vocab == c["vocab"] and got.cfg.max_seq == c["max_seq"]
    toks = [3, 17, 42, 5, 88, 0, 61]
    np.testing.assert_array_equal(got.forward(toks), ref.forward(toks))
    np.testing.assert_array_equal(got.forward_decode(9, len(toks)), ref.forward_decode(9, len(toks)))
    assert np.isfinite(got.forward(toks)).all()


@pytest.mark.gpu
def test_model_load_tensor_shape_errors(mri, gpu_ctx, oracle, tmp_path):
    c = TINY
    cfg = mri.LlamaConfig(c["n_layers"], c["dim"], c["n_heads"], c["ffn_dim"], c["vocab"], c["max_seq"],
                          n_kv_heads=c["n_kv_heads"])
    m = mri.LlamaModelInt8(cfg, ctx=gpu_ctx)
    raw = np.zeros(c["dim"] * 4, np.uint8)
    lib = m._lib
    # attn_q wants [128, 128]; a [1, 128] tensor is a shape mismatch.
    assert lib.mri_llama_load_tensor(m.handle, 3, 0, gguf.F32, raw.ctypes.data, raw.size, 1, c["dim"]) == 2
    # layer out of range, unknown role, unsupported type
    assert lib.mri_llama_load_tensor(m.handle, 7, 5, gguf.F32, raw.ctypes.data, raw.size, 1, c["dim"]) == 1
    assert lib.mri_llama_load_tensor(m.handle, 99, 0, gguf.F32, raw.ctypes.data, raw.size, 1, c["dim"]) == 6
    assert lib.mri_llama_load_tensor(m.handle, 7, 0, 3, raw.ctypes.data, raw.size, 1, c["dim"]) == 6
    assert lib.mri_llama_load_tensor(m.handle, 7, 0, gguf.F32, raw.ctypes.data, raw.size, 1, c["dim"]) == 0


def test_loader_module_is_importable_without_gpu():
    mri = load_mri()
    assert hasattr(mri.LlamaModelInt8, "from_gguf") and hasattr(mri.QuantizedMatrix, "from_gguf")
