"""GGUF container reader (and a small writer) for loading LlamaModelInt8 weights.

Host-side file parsing only: tensor data is handed to the device loader
(`mri_llama_load_tensor` / `mri_qmatrix_from_gguf`) as raw bytes of the mapped
file, and the dequantize + per-channel requantize of `from_loader` runs there.

Follows the reference's gguf module:
  header        src/gguf/header.rs:15-18, 58-95  (magic "GGUF", versions 2 and 3,
                u64 tensor and metadata counts)
  strings       header.rs:295-312                (u64 length, at most 1 MiB)
  metadata      src/gguf/metadata.rs:145-240, 440-465 (typed values, one level of
                arrays of at most 1e8 elements, bool 0/1, no duplicate keys,
                at most 100 000 entries)
  tensor infos  src/gguf/tensor_info.rs:71-110, 222-250 (name, n_dims <= 8, u64
                dims innermost first, ggml type, offset; no duplicate names)
  data section  src/gguf/loader.rs:114-150, 317-323; tensor_info.rs:372-379
                (aligned to general.alignment, default 32)
  type sizes    src/gguf/dtype.rs:140-200
  LlamaConfig   src/model/llama/config.rs:66-150
  tensor names  src/model/llama/weights.rs:62-104
"""
import mmap
import os
import struct

import numpy as np

GGUF_MAGIC = b"GGUF"
SUPPORTED_VERSIONS = (2, 3)
DEFAULT_ALIGNMENT = 32

# ggml type id -> (name, elements per block, bytes per block)  (dtype.rs:30-200)
GGML_TYPES = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20),
    6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 40),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144),
    13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 15: ("Q8_K", 256, 292),
    16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74), 18: ("IQ3_XXS", 256, 98),
    19: ("IQ1_S", 256, 50), 20: ("IQ4_NL", 256, 136), 21: ("IQ3_S", 256, 110),
    22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136), 24: ("I8", 1, 1), 25: ("I16", 1, 2), 26: ("I32", 1, 4), 27: ("I64", 1, 8),
    28: ("F64", 1, 8), 29: ("BF16", 1, 2),
}
F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8

# Metadata value types (metadata.rs GgufValueType).
(UINT8, INT8, UINT16, INT16, UINT32, INT32, FLOAT32, BOOL, STRING, ARRAY, UINT64, INT64,
 FLOAT64) = range(13)
_SCALAR = {UINT8: "<B", INT8: "<b", UINT16: "<H", INT16: "<h", UINT32: "<I", INT32: "<i",
           FLOAT32: "<f", UINT64: "<Q", INT64: "<q", FLOAT64: "<d"}


# ── errors (src/gguf/error.rs:7-60; src/model/mod.rs ModelError) ────────────

class GgufError(Exception):
    pass


class InvalidMagic(GgufError):
    pass


class UnsupportedVersion(GgufError):
    pass


class UnexpectedEof(GgufError):
    pass


class UnknownValueType(GgufError):
    pass


class InvalidBool(GgufError):
    pass


class NestedArray(GgufError):
    pass


class Overflow(GgufError):
    pass


class DuplicateKey(GgufError):
    pass


class ValueOutOfRange(GgufError):
    pass


class KeyNotFound(GgufError):
    pass


class TypeMismatch(GgufError):
    pass


class TensorDataUnavailable(GgufError):
    pass


class ModelError(Exception):
    pass


class MissingMetadataKey(ModelError):
    pass


class InvalidConfig(ModelError):
    pass


# ── reading ──────────────────────────────────────────────────────────────────

class _Cursor:
    def __init__(self, buf):
        self.buf = buf
        self.pos = 0

    def take(self, n, context):
        if self.pos + n > len(self.buf):
            raise UnexpectedEof(context)
        b = self.buf[self.pos:self.pos + n]
        self.pos += n
        return b

    def scalar(self, fmt, context):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt), context))[0]

    def string(self, context):
        n = self.scalar("<Q", context)
        if n > 1024 * 1024:
            raise Overflow(context)
        return bytes(self.take(n, context)).decode("utf-8", errors="replace")


def _read_value(cur, vtype, in_array=False):
    if vtype in _SCALAR:
        return cur.scalar(_SCALAR[vtype], "metadata value")
    if vtype == BOOL:
        b = cur.scalar("<B", "bool value")
        if b > 1:
            raise InvalidBool(b)
        return bool(b)
    if vtype == STRING:
        return cur.string("string value")
    if vtype == ARRAY:
        if in_array:
            raise NestedArray()
        etype = cur.scalar("<I", "array element type")
        if etype > FLOAT64:
            raise UnknownValueType(etype)
        n = cur.scalar("<Q", "array length")
        if n > 100_000_000:
            raise Overflow("array length")
        if etype in _SCALAR:
            fmt = _SCALAR[etype]
            size = struct.calcsize(fmt)
            raw = cur.take(n * size, "array element")
            return (etype, np.frombuffer(bytes(raw), dtype=np.dtype(fmt)).tolist())
        return (etype, [_read_value(cur, etype, True) for _ in range(n)])
    raise UnknownValueType(vtype)


class Metadata:
    """Key -> (value type, value); arrays are (element type, list)."""

    def __init__(self, entries=None):
        self.entries = dict(entries or {})

    def __len__(self):
        return len(self.entries)

    def __contains__(self, key):
        return key in self.entries

    def get(self, key):
        return self.entries.get(key)

    def get_u32(self, key):
        """metadata.rs:308-315: u8 / u16 / u32 values."""
        e = self.entries.get(key)
        return e[1] if e and e[0] in (UINT8, UINT16, UINT32) else None

    def get_u64(self, key):
        e = self.entries.get(key)
        return e[1] if e and e[0] in (UINT8, UINT16, UINT32, UINT64) else None

    def get_f32(self, key):
        e = self.entries.get(key)
        return e[1] if e and e[0] == FLOAT32 else None

    def get_string(self, key):
        e = self.entries.get(key)
        return e[1] if e and e[0] == STRING else None

    def get_string_array(self, key):
        e = self.entries.get(key)
        if e and e[0] == ARRAY and e[1][0] == STRING:
            return e[1][1]
        return None


class TensorInfo:
    def __init__(self, name, dims, dtype, offset):
        self.name, self.dims, self.dtype, self.offset = name, tuple(dims), dtype, offset

    @property
    def numel(self):
        n = 1
        for d in self.dims:
            n *= d
        return n

    def shape_row_major(self):
        """tensor_info.rs:145-147: GGUF dims are innermost first."""
        return tuple(reversed(self.dims))

    def size_bytes(self):
        _, block, size = GGML_TYPES[self.dtype]
        return self.numel // block * size

    @property
    def type_name(self):
        return GGML_TYPES[self.dtype][0]


def align_offset(offset, alignment):
    r = offset % alignment
    return offset if r == 0 else offset + (alignment - r)


def _read_header(cur):
    magic = bytes(cur.take(4, "magic"))
    if magic != GGUF_MAGIC:
        raise InvalidMagic(magic)
    version = cur.scalar("<I", "version")
    if version not in SUPPORTED_VERSIONS:
        raise UnsupportedVersion(version)
    return version, cur.scalar("<Q", "tensor count"), cur.scalar("<Q", "metadata count")


def read_header(data):
    """GgufHeader::read (header.rs:58-95): (version, tensor count, metadata
    count) from the first 24 bytes."""
    return _read_header(_Cursor(memoryview(bytes(data))))


class GgufFile:
    """GgufLoader::open (loader.rs:100-150): the file is memory-mapped and its
    header, metadata and tensor table parsed; tensor data stays in the map."""

    def __init__(self, path):
        self.path = os.fspath(path)
        with open(self.path, "rb") as f:
            size = os.fstat(f.fileno()).st_size
            self._map = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) if size else b""
        self._parse(memoryview(self._map))

    @classmethod
    def from_bytes(cls, data):
        self = cls.__new__(cls)
        self.path = "<bytes>"
        self._map = bytes(data)
        self._parse(memoryview(self._map))
        return self

    def _parse(self, view):
        cur = _Cursor(view)
        self.version, n_tensors, n_kv = _read_header(cur)
        if n_kv > 100_000:
            raise Overflow("metadata count")
        entries = {}
        for _ in range(n_kv):
            key = cur.string("metadata key")
            vtype = cur.scalar("<I", "value type")
            if vtype > FLOAT64:
                raise UnknownValueType(vtype)
            value = _read_value(cur, vtype)
            if key in entries:
                raise DuplicateKey(key)
            entries[key] = (vtype, value)
        self.metadata = Metadata(entries)
        if n_tensors > 100_000:
            raise ValueOutOfRange(f"tensor count {n_tensors}")
        self.tensors = {}
        self.tensor_order = []
        for _ in range(n_tensors):
            name = cur.string("tensor name")
            n_dims = cur.scalar("<I", "tensor n_dims")
            if n_dims > 8:
                raise ValueOutOfRange(f"tensor n_dims {n_dims}")
            dims = [cur.scalar("<Q", "tensor dimension") for _ in range(n_dims)]
            dtype = cur.scalar("<I", "tensor type")
            if dtype not in GGML_TYPES:
                raise UnknownValueType(dtype)  # GgmlType::from_u32 (dtype.rs:94-125)
            offset = cur.scalar("<Q", "tensor offset")
            if name in self.tensors:
                raise KeyNotFound(f"duplicate tensor name: {name}")
            self.tensors[name] = TensorInfo(name, dims, dtype, offset)
            self.tensor_order.append(name)
        self.alignment = self.metadata.get_u32("general.alignment") or DEFAULT_ALIGNMENT
        self.data_offset = align_offset(cur.pos, self.alignment)
        self._view = view

    def tensor(self, name):
        info = self.tensors.get(name)
        if info is None:
            raise KeyNotFound(name)
        return info

    def tensor_data(self, name):
        """loader.rs:202-224: the tensor's bytes as a read-only uint8 array, or
        None when they lie outside the file."""
        info = self.tensor(name)
        start = self.data_offset + info.offset
        end = start + info.size_bytes()
        if end > len(self._view):
            return None
        return np.frombuffer(self._view[start:end], dtype=np.uint8)

    def close(self):
        self._view = None
        if isinstance(self._map, mmap.mmap):
            self._map.close()


# ── LlamaConfig::from_metadata (model/llama/config.rs:66-150) ───────────────

def _u32_wide(meta, key):
    v = meta.get_u32(key)
    if v is None:
        v = meta.get_u64(key)
        if v is not None and v >= 1 << 32:
            v = None
    return v


def llama_config(meta):
    """Returns a dict of the LlamaConfig fields; raises MissingMetadataKey /
    InvalidConfig like the reference."""
    req = {}
    for field, key in (("block_count", "llama.block_count"),
                       ("embedding_length", "llama.embedding_length"),
                       ("n_heads", "llama.attention.head_count"),
                       ("feed_forward_length", "llama.feed_forward_length"),
                       ("context_length", "llama.context_length")):
        v = _u32_wide(meta, key)
        if v is None:
            raise MissingMetadataKey(key)
        req[field] = v
    n_kv = _u32_wide(meta, "llama.attention.head_count_kv")
    req["n_kv_heads"] = req["n_heads"] if n_kv is None else n_kv
    vocab = _u32_wide(meta, "llama.vocab_size")
    if vocab is None:
        toks = meta.get_string_array("tokenizer.ggml.tokens")
        if toks is None:
            raise MissingMetadataKey("llama.vocab_size")
        vocab = len(toks)
    req["vocab_size"] = vocab
    base = meta.get_f32("llama.rope.freq_base")
    req["rope_freq_base"] = 10000.0 if base is None else base
    eps = meta.get_f32("llama.attention.layer_norm_rms_epsilon")
    req["rms_norm_eps"] = 1e-5 if eps is None else eps
    h, d, kv = req["n_heads"], req["embedding_length"], req["n_kv_heads"]
    if h == 0:
        raise InvalidConfig("n_heads must be > 0")
    if d % h:
        raise InvalidConfig(f"embedding_length {d} not divisible by n_heads {h}")
    if kv == 0 or h % kv:
        raise InvalidConfig(f"n_heads {h} not divisible by n_kv_heads {kv}")
    return req


# weight_name / global_weight_name (model/llama/weights.rs:62-104), with the
# role ids of mri_llama_load_tensor.
GLOBAL_TENSORS = (("token_embd.weight", 0), ("output_norm.weight", 1), ("output.weight", 2))
LAYER_TENSORS = (("attn_q.weight", 3), ("attn_k.weight", 4), ("attn_v.weight", 5),
                 ("attn_output.weight", 6), ("attn_norm.weight", 7), ("ffn_gate.weight", 8),
                 ("ffn_up.weight", 9), ("ffn_down.weight", 10), ("ffn_norm.weight", 11))


def weight_name(layer, suffix):
    return f"blk.{layer}.{suffix}"


# ── writing (synthetic model files and tests) ───────────────────────────────

def _value_bytes(vtype, value):
    if vtype in _SCALAR:
        return struct.pack(_SCALAR[vtype], value)
    if vtype == BOOL:
        return struct.pack("<B", 1 if value else 0)
    if vtype == STRING:
        b = value.encode()
        return struct.pack("<Q", len(b)) + b
    if vtype == ARRAY:
        etype, items = value
        return struct.pack("<IQ", etype, len(items)) + b"".join(_value_bytes(etype, v) for v in items)
    raise UnknownValueType(vtype)


def write_gguf(path, metadata, tensors, version=3, alignment=DEFAULT_ALIGNMENT):
    """metadata: {key: (value type, value)}; tensors: list of (name,
    row-major shape, ggml type, raw bytes).  Writes a GGUF v2/v3 file."""
    out = bytearray(GGUF_MAGIC)
    out += struct.pack("<IQQ", version, len(tensors), len(metadata))
    for key, (vtype, value) in metadata.items():
        out += _value_bytes(STRING, key) + struct.pack("<I", vtype) + _value_bytes(vtype, value)
    offset = 0
    placed = []
    for name, shape, dtype, raw in tensors:
        raw = bytes(raw)
        dims = list(reversed([int(s) for s in shape]))
        out += _value_bytes(STRING, name) + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", dtype, offset)
        placed.append((offset, raw))
        offset = align_offset(offset + len(raw), alignment)
    out += b"\0" * (align_offset(len(out), alignment) - len(out))
    base = len(out)
    for off, raw in placed:
        out += b"\0" * (base + off - len(out))
        out += raw
    with open(path, "wb") as f:
        f.write(out)
