"""GGUF reader parity: the product's C++ reader (through the C ABI) against the
reference's own reader unit tests (src/reader.rs:308-359), the error variants
of src/error.rs, and the Python restatement in oracle/gguf_ref.py."""
import struct

import numpy as np
import pytest

from gguf_build import (ARRAY, BOOL, F32, I8, LLAMA_META, STRING, U32, U64, gstr, image, kv,
                        q8_bytes)


def _err(tirlib, fn, *args):
    with pytest.raises(tirlib.TirError) as e:
        fn(*args)
    return e.value


# ---- src/reader.rs:308-359 ---------------------------------------------------
def test_parse_general_u32(tirlib):
    data = struct.pack("<Q", 1) + b"n" + struct.pack("<I", 4) + struct.pack("<I", 22)
    fields, end = tirlib.GGUF.parse_general(data, 0, 1)
    assert fields == [("n", U32, 22)]
    assert end == len(data)


def test_parse_general_bool_is_one_byte(tirlib):
    data = struct.pack("<Q", 1) + b"b" + struct.pack("<I", 7) + bytes([1])
    fields, end = tirlib.GGUF.parse_general(data, 0, 1)
    assert fields == [("b", BOOL, True)]
    assert end == len(data)


def test_parse_general_truncated(tirlib):
    data = struct.pack("<Q", 100) + b"n"
    e = _err(tirlib, tirlib.GGUF.parse_general, data, 0, 1)
    assert e.name == "UNEXPECTED_EOF"
    assert e.message == "unexpected end of file reading string bytes at offset 8"


def test_parse_q8_block(tirlib):
    e = _err(tirlib, tirlib.parse_q8, 33, 34, 1024, 0)
    assert e.name == "BAD_QUANT_BLOCK"
    assert e.message == "q8_0 tensor length 33 is not a multiple of 32"
    assert tirlib.parse_q8(64, 34, 1024, 0) == 68
    assert _err(tirlib, tirlib.parse_q8, 64, 34, 67, 0).name == "UNEXPECTED_EOF"


# ---- whole files vs the Python restatement -----------------------------------
def _ref_kind(data):
    from oracle import gguf_ref
    try:
        gguf_ref.load_model(memoryview(data))
    except (gguf_ref.ReaderError, gguf_ref.MetaDataError, gguf_ref.ModelLoadError) as e:
        return e.kind
    return None


def _small_model_bytes(**kw):
    tens = [("token_embd.weight", 8, [64, 4], q8_bytes(256, 1)),
            ("blk.0.attn_norm.weight", 0, [64], np.ones(64, np.float32).tobytes())]
    return image(tensors=tens, **kw)


def test_tiny_synthetic_model_matches_oracle_reader(tirlib, tiny_path):
    from oracle import gguf_ref
    ours = tirlib.GGUF.open(tiny_path)
    ref = gguf_ref.GGUF(tiny_path)
    t = ours.transformer()
    rt = ref.transformer()
    for k in ("layers", "embed_dim", "q_heads", "k_v_heads", "dim"):
        assert t[k] == rt[k]
    assert t["base_freq"] == rt["base_freq"]
    meta = ours.metadata()
    assert [(n, v) for n, v, _ in meta] == [(n, v) for n, v, _ in ref.fields]
    for (n, vt, val), (_, _, rval) in zip(meta, ref.fields):
        if vt == F32:
            assert np.float32(val) == np.float32(rval)
        else:
            assert val == rval
    tens = ours.tensors()
    assert [(x["name"], x["shape"], x["dtype"], x["offset"], x["n_elements"]) for x in tens] == \
        [(x["name"], x["shape"], x["dtype"], x["offset"], x["n_elements"]) for x in ref.tensors]
    for name in ("token_embd.weight", "blk.1.ffn_down.weight", "output_norm.weight"):
        np.testing.assert_array_equal(ours.tensor_bytes(name), ref.tensor_bytes(name))
    e = _err(tirlib, ours.tensor_bytes, "blk.9.attn_q.weight")
    assert e.name == "TENSOR_LOAD" and e.message == "unable to load tensor: blk.9.attn_q.weight"


def test_minimal_model_parses(tirlib):
    g = tirlib.GGUF.from_bytes(_small_model_bytes())
    assert g.version() == 3
    assert [t["name"] for t in g.tensors()] == ["token_embd.weight", "blk.0.attn_norm.weight"]
    assert g.tensors()[0]["data_bytes"] == 8 * 34
    assert _ref_kind(_small_model_bytes()) is None


CASES = {
    "short_header": (lambda: b"GGUF" + b"\0" * 10, "UNEXPECTED_EOF", "UnexpectedEof",
                     "Reader Error: unexpected end of file reading gguf header at offset 14"),
    "bad_magic": (lambda: _small_model_bytes(magic=b"GGML"), "BAD_MAGIC", "BadMagic",
                  "Reader Error: bad magic number, not a gguf file"),
    "version_1": (lambda: _small_model_bytes(version=1), "BAD_VERSION", "BadVersion",
                  "Reader Error: unsupported gguf version: 1"),
    "version_4": (lambda: _small_model_bytes(version=4), "BAD_VERSION", "BadVersion",
                  "Reader Error: unsupported gguf version: 4"),
    "missing_layers": (lambda: image(meta=[m for m in LLAMA_META if m[0] != "llama.block_count"]),
                       "MISSING_FIELD", "MissingField",
                       "Metadata Load error: missing required field: Layers"),
    "wrong_type_is_missing": (lambda: image(meta=[(n, U64, v) if n == "llama.block_count" else (n, t, v)
                                                  for n, t, v in LLAMA_META]),
                              "MISSING_FIELD", "MissingField",
                              "Metadata Load error: missing required field: Layers"),
    "rope_base_as_u32": (lambda: image(meta=[(n, U32, 10000) if n == "llama.rope.freq_base" else (n, t, v)
                                             for n, t, v in LLAMA_META]),
                         "MISSING_FIELD", "MissingField",
                         "Metadata Load error: missing required field: Rope Base Frequency"),
    "unsupported_scalar": (lambda: b"GGUF" + struct.pack("<IQQ", 3, 0, 2) + kv(*LLAMA_META[0])
                           + gstr("x") + struct.pack("<I", 13),
                           "UNSUPPORTED_TYPE", "UnsupportedType",
                           "Reader Error: unsupported metadata value type: 13"),
    # arrays of arrays come back as UnsupportedType(9) (src/reader.rs:140)
    "nested_array": (lambda: b"GGUF" + struct.pack("<IQQ", 3, 0, 2) + kv(*LLAMA_META[0]) + gstr("arr")
                     + struct.pack("<IIQ", 9, 9, 1) + struct.pack("<IQ", 4, 0),
                     "UNSUPPORTED_TYPE", "UnsupportedType",
                     "Reader Error: unsupported metadata value type: 9"),
    "invalid_utf8": (lambda: b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + gstr(b"\xff\xfe") +
                     struct.pack("<I", 4) + struct.pack("<I", 1),
                     "INVALID_UTF8", "InvalidUtf8", "Reader Error: invalid utf8 in string at offset 32"),
    "truncated_tensor_data": (lambda: _small_model_bytes()[:-40], "TENSOR_DATA", "TensorDataError",
                              None),
    "unsupported_dtype": (lambda: image(tensors=[("t", 2, [32], b"\0" * 18)]), "TENSOR_DATA",
                          "TensorDataError",
                          "Tensor Weight Data Load Error: t: unsupported tensor dtype: 2"),
    "q8_not_multiple_of_32": (lambda: image(tensors=[("t", 8, [33], b"\0" * 68)]), "TENSOR_DATA",
                              "TensorDataError",
                              "Tensor Weight Data Load Error: t: q8_0 tensor length 33 is not a multiple of 32"),
    "truncated_tensor_info": (lambda: b"GGUF" + struct.pack("<IQQ", 3, 1, len(LLAMA_META))
                              + b"".join(kv(*m) for m in LLAMA_META) + gstr("t") + struct.pack("<I", 1)
                              + b"\0" * 4, "UNEXPECTED_EOF", "UnexpectedEof", None),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_error_variants(tirlib, case):
    make, status, ref_kind, msg = CASES[case]
    data = make()
    e = _err(tirlib, tirlib.GGUF.from_bytes, data)
    assert e.name == status, e.message
    if msg is not None:
        assert e.message == msg
    assert _ref_kind(data) == ref_kind


def test_metadata_values_roundtrip(tirlib):
    meta = LLAMA_META + [("s", STRING, "héllo"), ("b", BOOL, 0), ("i8", I8, -5),
                         ("arr", ARRAY, (U32, [1, 2, 3])), ("sarr", ARRAY, (STRING, ["a", "bc"])),
                         ("general.alignment", U32, 64)]
    g = tirlib.GGUF.from_bytes(image(meta=meta, tensors=[("t", 0, [4], np.arange(4, dtype=np.float32).tobytes())],
                                     alignment=64))
    got = {n: (t, v) for n, t, v in g.metadata()}
    assert got["s"] == (STRING, "héllo")
    assert got["b"] == (BOOL, False)
    assert got["i8"] == (I8, -5)
    assert got["arr"] == (ARRAY, (U32, [1, 2, 3]))
    assert got["sarr"] == (ARRAY, (STRING, ["a", "bc"]))
    np.testing.assert_array_equal(g.tensor_bytes("t").view(np.float32), np.arange(4, dtype=np.float32))


def test_open_missing_file(tirlib, tmp_path):
    e = _err(tirlib, tirlib.GGUF.open, str(tmp_path / "nope.gguf"))
    assert e.name == "IO"


def test_model_load_rejects_bad_file_before_touching_a_device(tirlib, tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"NOTAGGUF" * 8)
    e = _err(tirlib, tirlib.Model, str(p))
    assert e.name == "BAD_MAGIC"
