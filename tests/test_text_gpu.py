"""The text drivers on the GPU decode path: generate_capped and generate on
text (src/lib.rs:140-314) through tir_generate_capped_text / tir_generate_text,
against the oracle's model with the plain-Python tokenizer restatement (greedy
ids identical wherever the oracle's top-2 margin exceeds 1e-3)."""
import pytest

from oracle import tokenizer_ref as ref
from tir import synth
from test_decode_gpu import compare_tokens, oracle_greedy

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def text_model(cuda, tirlib, orc, small_path):
    from oracle.gguf_ref import GGUF
    g = tirlib.GGUF.open(small_path)
    tk = tirlib.Tokenizer.from_gguf(g)
    m = tirlib.Model(small_path)
    vocab, merges = synth.synthetic_tokenizer(synth.PRESETS["small"]["vocab"])
    yield m, tk, orc.model(GGUF(small_path)), vocab, merges
    m.close()
    tk.close()
    g.close()


@pytest.mark.parametrize("text", ["the rain in the hills", "ab  cd é 😀", ""])
def test_generate_capped_text(text_model, orc, text):
    m, tk, om, vocab, merges = text_model
    cap = 20
    st = m.state(max_ctx=128)
    got = st.generate_capped_text(tk, text, cap)
    prompt = ref.encode(vocab, merges, text)
    assert tk.encode(text).tolist() == prompt
    want, margins, _ = oracle_greedy(orc, om, prompt, cap)
    compare_tokens(got, want, margins)
    st.close()


def test_generate_text_stops_at_newline_or_eos(text_model):
    """generate keeps the greedy ids before the first 13 or 2 and decodes them."""
    m, tk, _, _, _ = text_model
    st = m.state(max_ctx=128)
    text = "she said hi"
    full = st.generate_capped_text(tk, text, 40).tolist()
    kept = []
    for t in full:
        if t in (13, 2):
            break
        kept.append(t)
    out, n = st.generate_text(tk, text, 40)
    assert n == len(kept)
    assert out == tk.decode(kept)
    st.close()


def test_generate_text_matches_oracle(text_model, orc):
    m, tk, om, vocab, merges = text_model
    st = m.state(max_ctx=128)
    text = "one more time"
    out, n = st.generate_text(tk, text, 24)
    ref_text, ref_ids, margins = ref.generate_text(om, vocab, merges, text, 24, orc.sample)
    got_ids = st.generate_capped_text(tk, text, n).tolist() if n else []
    if compare_tokens(got_ids, ref_ids[:n], margins) == min(n, len(ref_ids)) and n == len(ref_ids):
        assert out == ref_text
    st.close()
