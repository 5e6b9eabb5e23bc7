"""GGUF reader restated in Python -- TEST INFRASTRUCTURE ONLY.

Restates ``src/reader.rs`` (bounds-checked parser) and the parsing half of
``src/lib.rs:29-138`` ``load_model``.  Used as the checker for the product's
C++ reader and to hand raw tensor bytes to the C oracle.
"""
import mmap
import struct

import numpy as np

# src/state.rs:28-56 GgufMetadataValueType
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)


class ReaderError(Exception):
    """src/error.rs:5-24 ReaderError; ``kind`` is the variant name."""

    def __init__(self, kind, *args):
        super().__init__(kind, *args)
        self.kind = kind
        self.args_ = args


class MetaDataError(Exception):
    """src/error.rs:27-36 (MissingField)."""

    def __init__(self, kind, field):
        super().__init__(kind, field)
        self.kind = kind
        self.field = field


class ModelLoadError(Exception):
    """src/error.rs:47-57 TensorDataError."""

    def __init__(self, msg):
        super().__init__(msg)
        self.kind = "TensorDataError"


# src/reader.rs:25-37 take
def take(buf, offset, length, what):
    end = offset + length
    if end > len(buf) or offset > len(buf):
        raise ReaderError("UnexpectedEof", what, offset)
    return buf[offset:end]


def _read_u32(buf, off, what):
    return struct.unpack_from("<I", take(buf, off, 4, what))[0], off + 4


def _read_u64(buf, off, what):
    return struct.unpack_from("<Q", take(buf, off, 8, what))[0], off + 8


_SCALAR = {U8: ("<B", 1), I8: ("<b", 1), U16: ("<H", 2), I16: ("<h", 2), U32: ("<I", 4),
           I32: ("<i", 4), F32: ("<f", 4), BOOL: ("<B", 1), U64: ("<Q", 8), I64: ("<q", 8),
           F64: ("<d", 8)}
_NAMES = {U8: "u8", I8: "i8", U16: "u16", I16: "i16", U32: "u32", I32: "i32", F32: "f32",
          BOOL: "bool", U64: "u64", I64: "i64", F64: "f64"}


# src/reader.rs:50-96 read_scalar
def read_scalar(buf, off, vtype):
    if vtype not in _SCALAR:
        raise ReaderError("UnsupportedType", vtype)
    fmt, width = _SCALAR[vtype]
    v = struct.unpack_from(fmt, take(buf, off, width, _NAMES[vtype]))[0]
    if vtype == BOOL:
        v = v != 0
    return v, off + width


# src/reader.rs:191-199 parse_string
def parse_string(buf, off):
    length, off = _read_u64(buf, off, "string length")
    raw = bytes(take(buf, off, length, "string bytes"))
    try:
        s = raw.decode("utf-8")
    except UnicodeDecodeError:
        raise ReaderError("InvalidUtf8", off)
    return s, off + length


# src/reader.rs:98-169 parse_general: returns [(name, vtype, value)], offset
def parse_general(buf, off, count):
    info = []
    while count != 0:
        name, off = parse_string(buf, off)
        ftype, off = _read_u32(buf, off, "field type")
        if ftype == STRING:
            v, off = parse_string(buf, off)
            info.append((name, STRING, v))
        elif ftype == ARRAY:
            etype, off = _read_u32(buf, off, "array element type")
            n, off = _read_u64(buf, off, "array length")
            vals = []
            for _ in range(n):
                if etype == STRING:
                    v, off = parse_string(buf, off)
                else:
                    v, off = read_scalar(buf, off, etype)
                vals.append(v)
            info.append((name, ARRAY, (etype, vals)))
        else:
            v, off = read_scalar(buf, off, ftype)
            info.append((name, ftype, v))
        count -= 1
    return info, off


# src/reader.rs:201-238 parse_tensors: returns [dict], offset
def parse_tensors(buf, off, count):
    tensors = []
    while count != 0:
        name, off = parse_string(buf, off)
        ndim, off = _read_u32(buf, off, "tensor dimension count")
        shape = []
        for _ in range(ndim):
            v, off = _read_u64(buf, off, "tensor dimension")
            shape.append(v)
        dtype, off = _read_u32(buf, off, "tensor dtype")
        toff = struct.unpack_from("<Q", take(buf, off, 8, "tensor offset"))[0]
        tensors.append({"name": name, "shape": shape, "n_elements": ndim, "dtype": dtype,
                        "offset": toff})
        off += 8
        count -= 1
    return tensors, off


# src/reader.rs:258-272 parse_q8
def parse_q8(count, byte_count, buf, off):
    if count % 32 != 0:
        raise ReaderError("BadQuantBlock", count)
    return take(buf, off, (count // 32) * byte_count, "q8_0 tensor data")


# src/reader.rs:240-256 parse_tensor_data
def parse_tensor_data(buf, off, tensor):
    count = int(np.prod(tensor["shape"], dtype=np.uint64)) if tensor["shape"] else 1
    if tensor["dtype"] == 0:
        return take(buf, off, count * 4, "f32 tensor data")
    if tensor["dtype"] == 8:
        return parse_q8(count, 34, buf, off)
    raise ReaderError("UnsupportedDtype", tensor["dtype"])


# src/lib.rs:29-138 load_model (parsing; the product uploads instead of mmap)
def load_model(buf):
    if len(buf) < 24:
        raise ReaderError("UnexpectedEof", "gguf header", len(buf))
    if bytes(buf[:4]) != b"GGUF":
        raise ReaderError("BadMagic")
    version = struct.unpack_from("<I", buf, 4)[0]
    if not (2 <= version <= 3):
        raise ReaderError("BadVersion", version)
    n_tensors, n_kv = struct.unpack_from("<QQ", buf, 8)
    fields, off = parse_general(buf, 24, n_kv)
    want = {"llama.block_count": ("layers", U32), "llama.rope.dimension_count": ("dim", U32),
            "llama.embedding_length": ("embed_dim", U32),
            "llama.attention.head_count": ("q_heads", U32),
            "llama.attention.head_count_kv": ("k_v_heads", U32),
            "llama.rope.freq_base": ("base_freq", F32)}
    got = {}
    alignment = 32
    for name, vtype, value in fields:
        if name in want and want[name][1] == vtype:
            got[want[name][0]] = value
        elif name == "general.alignment" and vtype == U32:
            alignment = value
    for key, label in (("layers", "Layers"), ("dim", "Dimension"),
                       ("embed_dim", "Embedding Length"), ("q_heads", "Query Attention Heads"),
                       ("k_v_heads", "K/V Attention Heads"),
                       ("base_freq", "Rope Base Frequency")):
        if key not in got:
            raise MetaDataError("MissingField", label)
    tensors, off = parse_tensors(buf, off, n_tensors)
    data_start = -(-off // alignment) * alignment
    tmap = {}
    for t in tensors:
        try:
            tmap[t["name"]] = parse_tensor_data(buf, data_start + t["offset"], t)
        except ReaderError as e:
            raise ModelLoadError(f"{t['name']}: {e}")
    return got, fields, tensors, tmap


class GGUF:
    """A file (or bytes) parsed with ``load_model``; tensors as numpy views."""

    def __init__(self, path_or_bytes):
        if isinstance(path_or_bytes, (bytes, bytearray)):
            self._buf = memoryview(bytes(path_or_bytes))
        else:
            self._f = open(path_or_bytes, "rb")
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
            self._buf = memoryview(self._mm)
        self._transformer, self.fields, self.tensors, self._map = load_model(self._buf)
        self._shapes = {t["name"]: t["shape"] for t in self.tensors}

    def transformer(self):
        return dict(self._transformer)

    def tensor_shape(self, name):
        return self._shapes[name]

    def tensor_bytes(self, name):
        return np.frombuffer(self._map[name], dtype=np.uint8)

    def tensor_f32(self, name):
        return np.frombuffer(self._map[name], dtype=np.float32)
