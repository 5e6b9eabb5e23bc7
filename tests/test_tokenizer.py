"""BPE tokenizer (src/tokenizer.rs:37-150) through the C ABI, on the host (no
GPU): the reference's own known-answer cases (src/tokenizer.rs:168-235, its
mock vocab and merges), the synthetic GGUF's tokenizer fields, and randomized
text against the plain-Python restatement in oracle/tokenizer_ref.py."""
import numpy as np
import pytest

from oracle import tokenizer_ref as ref
from tir import synth

# src/tokenizer.rs:187-196: mock_vocab / mock_merges
MOCK_VOCAB = ["<unk>", "<s>", "</s>", "<0x21>", "▁", "a", "b", "▁a", "ab", "▁ab", "▁b"]
MOCK_MERGES = ["▁ a", "a b", "▁a b", "▁ b"]


@pytest.fixture(scope="module")
def mock(tirlib):
    t = tirlib.Tokenizer.from_lists(MOCK_VOCAB, MOCK_MERGES)
    yield t
    t.close()


@pytest.mark.parametrize("text,ids", [
    ("ab", [1, 9]),            # encode_merge_order_test: "▁ a" outranks "a b"
    ("a  b", [1, 7, 4, 10]),   # encode_whitespace_test: the double space survives as ▁
    ("a b!", [1, 7, 10, 3]),   # encode_byte_fallback_test: "!" only as <0x21>
])
def test_reference_encode_cases(mock, text, ids):
    assert mock.encode(text).tolist() == ids
    assert ref.encode(MOCK_VOCAB, MOCK_MERGES, text) == ids


def test_reference_round_trip(mock):
    """round_trip_test: skip BOS, the prefix space is the only artifact."""
    ids = mock.encode("a b!")
    assert mock.decode(ids[1:]) == " a b!"


def test_reference_unknown_id(tirlib, mock):
    """decode_unknown_id_test: id 999 is not in the vocab."""
    with pytest.raises(tirlib.TirError) as e:
        mock.decode([999])
    assert e.value.name == "BAD_TOKEN"
    assert "999" in str(e.value)


def test_decode_edge_cases(tirlib):
    vocab = ["<unk>", "<s>", "</s>", "<0xE2>", "<0x82>", "<0xAC>", "<0x+41>", "<0x100>", "<0x>", "x▁y", "<0xC3>"]
    t = tirlib.Tokenizer.from_lists(vocab, [])
    for ids in ([3, 4, 5], [3, 4], [6], [7, 8], [9], [10, 9], [3, 10, 5], []):
        assert t.decode(ids) == ref.decode(vocab, ids), ids
    assert t.decode([3, 4, 5]) == "€"           # byte tokens reassemble a char
    assert t.decode([6]) == "A"                 # from_str_radix accepts a leading '+'
    assert t.decode([7]) == "<0x100>"           # > 255: not a byte token
    assert t.decode([10, 9]) == "�x y"     # a lone lead byte is replaced
    t.close()


def test_repeated_tokens_and_merges_keep_the_last(tirlib):
    vocab = ["<unk>", "<s>", "</s>", "a", "b", "ab", "ab"]
    merges = ["a b", "x y", "a b"]
    t = tirlib.Tokenizer.from_lists(vocab, merges)
    assert t.encode("ab").tolist() == ref.encode(vocab, merges, "ab")
    t.close()


def test_synthetic_gguf_tokenizer(tirlib, tiny_path):
    g = tirlib.GGUF.open(tiny_path)
    t = tirlib.Tokenizer.from_gguf(g)
    vocab, merges = synth.synthetic_tokenizer(synth.PRESETS["tiny"]["vocab"])
    assert len(t) == len(vocab)
    for text in ["the cat sat", "  double  spaces ", "ünïcödé ☃ 😀", "", "aaaa tttt", "\n\t"]:
        assert t.encode(text).tolist() == ref.encode(vocab, merges, text), text
        ids = t.encode(text)
        assert t.decode(ids[1:]) == ref.decode(vocab, ids[1:].tolist())
    t.close()
    g.close()


def test_missing_and_mistyped_tokenizer_fields(tirlib):
    """The drivers' MissingField("ggml.tokens") (src/lib.rs:159) and encode's
    WrongType("array of tokens") (src/tokenizer.rs:42-44)."""
    import gguf_build as gb
    g = tirlib.GGUF.from_bytes(gb.image())
    with pytest.raises(tirlib.TirError) as e:
        tirlib.Tokenizer.from_gguf(g)
    assert e.value.name == "MISSING_FIELD" and "ggml.tokens" in str(e.value)
    g.close()
    g = tirlib.GGUF.from_bytes(gb.image(gb.LLAMA_META + [("tokenizer.ggml.tokens", gb.STRING, "x"),
                                                         ("tokenizer.ggml.merges", gb.ARRAY, (gb.STRING, []))]))
    with pytest.raises(tirlib.TirError) as e:
        tirlib.Tokenizer.from_gguf(g)
    assert e.value.name == "WRONG_TYPE" and "array of tokens" in str(e.value)
    g.close()


def test_randomized_against_restatement(tirlib):
    rng = np.random.default_rng(3)
    vocab, merges = synth.synthetic_tokenizer(2000)
    t = tirlib.Tokenizer.from_lists(vocab, merges)
    alphabet = list("etaoinshr abcxyz  ") + ["é", "ß", "中", "😀", "\n"]
    for _ in range(200):
        text = "".join(rng.choice(alphabet, size=int(rng.integers(0, 40))))
        ids = t.encode(text)
        assert ids.tolist() == ref.encode(vocab, merges, text), text
        assert t.decode(ids) == ref.decode(vocab, ids.tolist())
    t.close()


def test_invalid_utf8_input(tirlib, mock):
    with pytest.raises(tirlib.TirError) as e:
        mock.encode(b"a\xffb")
    assert e.value.name == "INVALID_UTF8"
