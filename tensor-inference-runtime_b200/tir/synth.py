"""Seeded synthetic Llama-2 models written as Q8_0 GGUF v3 files.

No checkpoint or dataset is available, so every model this runtime is tested
and measured on is generated here:

* linear weights: f32 N(0, 0.02) from numpy PCG64, one seed per tensor derived
  from a base seed and the tensor name, quantised to Q8_0 (blocks of 32 int8
  with an f16 scale): ``d = amax/127`` (f32), ``q = rint(x/d)`` clamped to
  [-127, 127], stored ``f16(d)``;
* norm weights: f32 ``1 + N(0, 0.01)``;
* ``token_embd.weight`` and ``output.weight``: Q8_0 ``[embed_dim, vocab]``.

The metadata keys are the ones the reference's ``load_model`` reads
(``src/lib.rs:78-97``, each with the wire type it requires) plus the keys a
llama GGUF normally carries.  Tensor shapes follow the GGUF convention
(``ne0`` first): a ``[K, N]`` Q8_0 tensor is N rows of K/32 blocks of 34 bytes.
"""
import os
import struct
import zlib

import numpy as np

GGUF_MAGIC = b"GGUF"
ALIGN = 32

PRESETS = {
    # TinyLlama-1.1B shape: the reference's only supported shape.
    "tinyllama": dict(n_layers=22, embed_dim=2048, q_heads=32, kv_heads=4, head_dim=64,
                      ffn_dim=5632, vocab=32000, rope_theta=10000.0, rms_eps=1e-5, ctx=2048),
    # Small shapes for fast parity tests (same code paths, fewer bytes).
    "small": dict(n_layers=4, embed_dim=1024, q_heads=16, kv_heads=4, head_dim=64,
                  ffn_dim=2816, vocab=4000, rope_theta=10000.0, rms_eps=1e-5, ctx=1024),
    "tiny": dict(n_layers=2, embed_dim=512, q_heads=8, kv_heads=2, head_dim=64,
                 ffn_dim=1408, vocab=1000, rope_theta=10000.0, rms_eps=1e-5, ctx=512),
}

_T_U32, _T_F32, _T_STRING, _T_ARRAY = 4, 6, 8, 9


def _rng(seed, name):
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, zlib.crc32(name.encode())])))


def quantize_q8_0(x):
    """f32 [rows, K] -> Q8_0 bytes [rows, K/32*34]."""
    rows, k = x.shape
    xb = x.reshape(rows, k // 32, 32)
    amax = np.abs(xb).max(axis=2)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(d[..., None] > 0, np.rint(xb / d[..., None]), 0.0)
    q = np.clip(q, -127, 127).astype(np.int8)
    out = np.empty((rows, k // 32, 34), np.uint8)
    out[..., :2] = d.astype(np.float16).view(np.uint8).reshape(rows, k // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(rows, k // 32 * 34)


def _q8_tensor(seed, name, k, n, std=0.02, chunk_rows=4096):
    rng = _rng(seed, name)
    parts = []
    for r0 in range(0, n, chunk_rows):
        r = min(chunk_rows, n - r0)
        x = rng.standard_normal((r, k), dtype=np.float32) * np.float32(std)
        parts.append(quantize_q8_0(x))
    return np.concatenate(parts, axis=0)


def _norm_tensor(seed, name, n):
    rng = _rng(seed, name)
    return (np.float32(1.0) + rng.standard_normal(n, dtype=np.float32) * np.float32(0.01)).astype(np.float32)


def _gguf_string(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def tensor_specs(cfg):
    """(name, dtype, shape [ne0, ne1...]) in file order."""
    H, F, V = cfg["embed_dim"], cfg["ffn_dim"], cfg["vocab"]
    KVD = cfg["kv_heads"] * cfg["head_dim"]
    specs = [("token_embd.weight", 8, [H, V])]
    for l in range(cfg["n_layers"]):
        p = f"blk.{l}."
        specs += [(p + "attn_norm.weight", 0, [H]), (p + "attn_q.weight", 8, [H, H]),
                  (p + "attn_k.weight", 8, [H, KVD]), (p + "attn_v.weight", 8, [H, KVD]),
                  (p + "attn_output.weight", 8, [H, H]), (p + "ffn_norm.weight", 0, [H]),
                  (p + "ffn_gate.weight", 8, [H, F]), (p + "ffn_up.weight", 8, [H, F]),
                  (p + "ffn_down.weight", 8, [F, H])]
    specs += [("output_norm.weight", 0, [H]), ("output.weight", 8, [H, V])]
    return specs


def _nbytes(dtype, shape):
    n = int(np.prod(shape))
    return n * 4 if dtype == 0 else n // 32 * 34


SPACE = "\u2581"  # sentencepiece's word-boundary mark


def synthetic_tokenizer(vocab):
    """A BPE vocabulary of `vocab` tokens and its merge list, shaped like a
    llama sentencepiece tokenizer: <unk>, <s>, </s>, the 256 byte tokens
    <0x00>..<0xFF>, the word mark, a-z, mark+letter, letter pairs, then
    filler pieces.  Synthetic: it exercises encode/decode and the text
    drivers, not any real language."""
    letters = [chr(c) for c in range(ord("a"), ord("z") + 1)]
    toks = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)] + [SPACE] + letters
    merges = []
    for l in letters:
        toks.append(SPACE + l)
        merges.append(f"{SPACE} {l}")
    for a in "etaoinshr":
        for b in "etaoinshr":
            toks.append(a + b)
            merges.append(f"{a} {b}")
            toks.append(SPACE + a + b)
            merges.append(f"{SPACE}{a} {b}")
    i = 0
    while len(toks) < vocab:
        toks.append(f"{SPACE}w{i}")
        i += 1
    return toks[:vocab], merges


def _gguf_string_array(values):
    return struct.pack("<IQ", _T_STRING, len(values)) + b"".join(_gguf_string(v) for v in values)


def write_gguf(path, cfg, seed=0):
    """Writes the synthetic model ``cfg`` (a PRESETS entry) to ``path``."""
    meta = [("general.architecture", _T_STRING, "llama"),
            ("general.name", _T_STRING, "synthetic-llama-q8_0"),
            ("general.alignment", _T_U32, ALIGN),
            ("llama.block_count", _T_U32, cfg["n_layers"]),
            ("llama.context_length", _T_U32, cfg["ctx"]),
            ("llama.embedding_length", _T_U32, cfg["embed_dim"]),
            ("llama.feed_forward_length", _T_U32, cfg["ffn_dim"]),
            ("llama.attention.head_count", _T_U32, cfg["q_heads"]),
            ("llama.attention.head_count_kv", _T_U32, cfg["kv_heads"]),
            ("llama.rope.dimension_count", _T_U32, cfg["head_dim"]),
            ("llama.rope.freq_base", _T_F32, cfg["rope_theta"]),
            ("llama.attention.layer_norm_rms_epsilon", _T_F32, cfg["rms_eps"]),
            ("general.file_type", _T_U32, 7)]
    toks, merges = synthetic_tokenizer(cfg["vocab"])
    meta += [("tokenizer.ggml.model", _T_STRING, "llama"),
             ("tokenizer.ggml.tokens", _T_ARRAY, toks),
             ("tokenizer.ggml.merges", _T_ARRAY, merges)]
    specs = tensor_specs(cfg)
    head = bytearray(GGUF_MAGIC + struct.pack("<IQQ", 3, len(specs), len(meta)))
    for name, t, v in meta:
        head += _gguf_string(name) + struct.pack("<I", t)
        if t == _T_U32:
            head += struct.pack("<I", v)
        elif t == _T_F32:
            head += struct.pack("<f", v)
        elif t == _T_ARRAY:
            head += _gguf_string_array(v)
        else:
            head += _gguf_string(v)
    offset = 0
    offsets = []
    for name, dtype, shape in specs:
        offsets.append(offset)
        head += _gguf_string(name) + struct.pack("<I", len(shape))
        head += b"".join(struct.pack("<Q", s) for s in shape)
        head += struct.pack("<IQ", dtype, offset)
        offset += -(-_nbytes(dtype, shape) // ALIGN) * ALIGN
    head += b"\0" * (-len(head) % ALIGN)
    tmp = f"{path}.partial.{os.getpid()}"  # ranks writing the same file never share a temp
    with open(tmp, "wb") as f:
        f.write(head)
        for (name, dtype, shape), off in zip(specs, offsets):
            if dtype == 0:
                data = _norm_tensor(seed, name, shape[0]).tobytes()
            else:
                data = _q8_tensor(seed, name, shape[0], shape[1]).tobytes()
            f.write(data)
            f.write(b"\0" * (-len(data) % ALIGN))
    os.replace(tmp, path)
    return path


def cache_dir():
    d = os.environ.get("TIR_MODEL_CACHE") or os.path.join(
        os.environ.get("TMPDIR", "/tmp"), "tir_models")
    os.makedirs(d, exist_ok=True)
    return d


def synthetic_model(preset="tinyllama", seed=0):
    """Path of the cached synthetic GGUF for (preset, seed), written on first use."""
    path = os.path.join(cache_dir(), f"{preset}-q8_0-seed{seed}-tok.gguf")
    if not os.path.exists(path):
        write_gguf(path, PRESETS[preset], seed)
    return path


def prompt_ids(n, vocab, seed=0):
    """Seeded uniform token ids in [3, vocab)."""
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, 0x70726F6D])))
    return rng.integers(3, vocab, size=n, dtype=np.int64).astype(np.int32)


def gemv_case(k, n, seed=0):
    """GEMV-sweep inputs: x f32 N(0,1); int8 weights uniform in [-127, 127];
    f16 scales |N(0, 0.02)|/127.  Returns (x, Q8_0 bytes [n, k/32*34])."""
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, k, n])))
    x = rng.standard_normal(k, dtype=np.float32)
    q = rng.integers(-127, 128, size=(n, k // 32, 32), dtype=np.int16).astype(np.int8)
    s = (np.abs(rng.standard_normal((n, k // 32), dtype=np.float32)) * np.float32(0.02)
         / np.float32(127.0)).astype(np.float16)
    blocks = np.empty((n, k // 32, 34), np.uint8)
    blocks[..., :2] = s.view(np.uint8).reshape(n, k // 32, 2)
    blocks[..., 2:] = q.view(np.uint8)
    return x, blocks.reshape(n, k // 32 * 34)
