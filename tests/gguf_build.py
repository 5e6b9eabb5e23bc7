"""Builds small GGUF images in memory for reader tests."""
import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
        U64: "<Q", I64: "<q", F64: "<d"}


def gstr(s):
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def value(vtype, v):
    if vtype == STRING:
        return gstr(v)
    if vtype == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(value(et, i) for i in items)
    return struct.pack(_FMT[vtype], v)


def kv(name, vtype, v):
    return gstr(name) + struct.pack("<I", vtype) + value(vtype, v)


LLAMA_META = [("general.architecture", STRING, "llama"), ("llama.block_count", U32, 1),
              ("llama.rope.dimension_count", U32, 64), ("llama.embedding_length", U32, 64),
              ("llama.attention.head_count", U32, 1), ("llama.attention.head_count_kv", U32, 1),
              ("llama.rope.freq_base", F32, 10000.0)]


def image(meta=None, tensors=(), version=3, alignment=32, magic=b"GGUF"):
    """tensors: [(name, dtype, shape, data_bytes)] laid out in order, aligned."""
    meta = LLAMA_META if meta is None else meta
    head = magic + struct.pack("<IQQ", version, len(tensors), len(meta))
    head += b"".join(kv(*m) for m in meta)
    off = 0
    datas = []
    for name, dtype, shape, data in tensors:
        head += gstr(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", s) for s in shape)
        head += struct.pack("<IQ", dtype, off)
        datas.append(data)
        off += -(-len(data) // alignment) * alignment
    head += b"\0" * (-len(head) % alignment)
    body = b"".join(d + b"\0" * (-len(d) % alignment) for d in datas)
    return head + body


def q8_bytes(n_weights, seed=0):
    rng = np.random.default_rng(seed)
    nb = n_weights // 32
    blocks = np.empty((nb, 34), np.uint8)
    blocks[:, :2] = (rng.uniform(0.001, 0.01, nb).astype(np.float16)).view(np.uint8).reshape(nb, 2)
    blocks[:, 2:] = rng.integers(-127, 128, (nb, 32)).astype(np.int8).view(np.uint8)
    return blocks.tobytes()
