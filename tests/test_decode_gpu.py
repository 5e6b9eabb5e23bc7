"""Whole-path parity on the GPU: the persistent decode kernel (through the C ABI)
against the oracle's restatement of src/forward.rs / src/lib.rs on identical
synthetic-GGUF weights and token ids.

Bars:
  * per-layer hidden states (residual stream) within fp32 relative-L2 1e-4;
  * greedy tokens identical wherever the oracle's top-2 logit margin > 1e-3
    (at the first mismatch the margin must be <= 1e-3; later tokens then have
    different contexts and are not compared).
"""
import numpy as np
import pytest

from tir import synth

pytestmark = pytest.mark.gpu

LAYER_TOL = 1e-4
MARGIN = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def models(cuda, tirlib, orc, tiny_path, small_path):
    from oracle.gguf_ref import GGUF
    out = {}
    for name, path in (("tiny", tiny_path), ("small", small_path)):
        out[name] = (tirlib.Model(path), orc.model(GGUF(path)))
    yield out
    for m, _ in out.values():
        m.close()


def oracle_greedy(orc, om, prompt, cap):
    """src/lib.rs:239-314 on the oracle, also returning each step's top-2 margin."""
    om.reset()
    logits = None
    pos = 0
    for t in prompt:
        logits = om.forward(om.embed(int(t)), pos)
        pos += 1
    ids, margins = [], []
    for _ in range(cap):
        srt = np.sort(logits)
        margins.append(float(srt[-1]) - float(srt[-2]))
        tok = orc.sample(logits)
        ids.append(tok)
        logits = om.forward(om.embed(tok), pos)
        pos += 1
    return np.array(ids, np.int32), margins, logits


def compare_tokens(got, ref, margins):
    """Returns how many leading tokens agree; asserts the margin rule."""
    for j, (a, b) in enumerate(zip(got, ref)):
        if a != b:
            assert margins[j] <= MARGIN, f"token {j}: gpu {a} != oracle {b} with oracle margin {margins[j]:.3g}"
            return j
    return len(ref)


@pytest.mark.parametrize("name", ["tiny", "small"])
def test_per_layer_hidden_states(models, name):
    m, om = models[name]
    st = m.state(max_ctx=64)
    st.enable_dump(True)
    om.reset()
    ids = synth.prompt_ids(6, m.info["vocab"], seed=1)
    for pos, t in enumerate(ids):
        x = om.embed(int(t))
        ref_logits, ref_dump = om.forward(x, pos, dump=True)
        logits = st.forward_embedded(x, pos)
        dump = st.dump()
        np.testing.assert_array_equal(dump[0], x)
        for l in range(1, dump.shape[0]):
            assert rel_l2(dump[l], ref_dump[l]) < LAYER_TOL, (pos, l, rel_l2(dump[l], ref_dump[l]))
        assert rel_l2(logits, ref_logits) < LAYER_TOL
    st.close()


def test_prefill_and_layer_dump(models, tirlib):
    """tir_prefill: the prompt pass alone (the logits generate_capped(prompt, 0)
    leaves, and the oracle's after the same ids); tir_debug_dump_layers: the
    layer outputs of the dump."""
    m, om = models["small"]
    ids = synth.prompt_ids(7, m.info["vocab"], seed=11)
    st = m.state(max_ctx=16)
    st.enable_dump(True)
    lg = st.prefill(ids)
    _, ref = st.generate_capped(ids, 0, want_logits=True)
    np.testing.assert_array_equal(lg, ref)
    np.testing.assert_array_equal(st.dump_layers(), st.dump()[1:])
    om.reset()
    for pos, t in enumerate(ids):
        want = om.forward(om.embed(int(t)), pos)
    assert rel_l2(lg, want) < LAYER_TOL
    with pytest.raises(tirlib.TirError) as e:
        tirlib.check(tirlib.lib().tir_prefill(st._h, ids.ctypes.data, 2, len(ids), None))
    assert e.value.name == "INVALID_ARG"
    st.close()


def test_forward_by_token_equals_embedded(models):
    m, om = models["tiny"]
    a, b = m.state(max_ctx=16), m.state(max_ctx=16)
    for pos, t in enumerate([5, 900, 3]):
        la = a.forward(t, pos)
        lb = b.forward_embedded(om.embed(t), pos)
        np.testing.assert_array_equal(la, lb)
    a.close()
    b.close()


@pytest.mark.parametrize("name,n_prompt,cap", [("tiny", 8, 24), ("small", 16, 48), ("small", 1, 8)])
def test_generate_capped_tokens(models, orc, name, n_prompt, cap):
    m, om = models[name]
    prompt = synth.prompt_ids(n_prompt, m.info["vocab"], seed=n_prompt)
    st = m.state(max_ctx=n_prompt + cap)
    got, logits = st.generate_capped(prompt, cap, want_logits=True)
    ref, margins, ref_logits = oracle_greedy(orc, om, prompt, cap)
    agree = compare_tokens(got, ref, margins)
    if agree == cap:
        assert rel_l2(logits, ref_logits) < LAYER_TOL
    assert len(st) == n_prompt + cap
    # deterministic: same call, same bits
    again, logits2 = st.generate_capped(prompt, cap, want_logits=True)
    np.testing.assert_array_equal(again, got)
    np.testing.assert_array_equal(logits2, logits)
    st.close()


def test_long_context_split_attention(models, orc):
    """Context up to 700 positions: the attention phase splits each KV head over
    up to 22 CTAs and combines partial softmaxes."""
    m, om = models["small"]
    prompt = synth.prompt_ids(690, m.info["vocab"], seed=77)
    cap = 10
    st = m.state(max_ctx=1024)
    got, logits = st.generate_capped(prompt, cap, want_logits=True)
    ref, margins, ref_logits = oracle_greedy(orc, om, prompt, cap)
    agree = compare_tokens(got, ref, margins)
    if agree == cap:
        assert rel_l2(logits, ref_logits) < LAYER_TOL
    st.close()


def test_test_forward(models, orc):
    m, om = models["small"]
    st = m.state(max_ctx=4)
    got = st.test_forward()
    om.reset()
    logits = om.forward(np.ones(m.info["embed_dim"], np.float32), 0)
    srt = np.sort(logits)
    if got != orc.sample(logits):
        assert srt[-1] - srt[-2] <= MARGIN
    st.close()


def test_state_errors(models):
    m, _ = models["tiny"]
    st = m.state(max_ctx=4)
    import tir
    with pytest.raises(tir.TirError) as e:
        st.forward(m.info["vocab"], 0)
    assert e.value.name == "BAD_TOKEN"
    with pytest.raises(tir.TirError) as e:
        st.forward(1, 3)
    assert e.value.name == "INVALID_ARG"
    with pytest.raises(tir.TirError) as e:
        st.generate_capped([1, 2, 3], 2)
    assert e.value.name == "CTX_OVERFLOW"
    with pytest.raises(tir.TirError) as e:
        st.generate_capped([1, -2], 1)
    assert e.value.name == "BAD_TOKEN"
    for pos in range(4):
        st.forward(1, pos)
    with pytest.raises(tir.TirError) as e:
        st.forward(1, 4)
    assert e.value.name == "CTX_OVERFLOW"
    st.reset()
    assert len(st) == 0
    st.forward(1, 0)
    st.close()


def test_empty_prompt_samples_token_zero(models, orc):
    """src/lib.rs:295: with no prompt the first sample is over empty logits -> 0."""
    m, om = models["tiny"]
    st = m.state(max_ctx=8)
    got = st.generate_capped(np.zeros(0, np.int32), 3)
    assert got[0] == 0
    ref = orc.sample([])
    assert ref == 0
    st.close()


def test_tinyllama_config0_slice(cuda, tirlib, orc, tinyllama_path):
    """TinyLlama-1.1B shape (22 layers, 2048/5632/32000): per-layer states of the
    first positions and 16 prompt + 32 greedy tokens against the oracle."""
    from oracle.gguf_ref import GGUF
    m = tirlib.Model(tinyllama_path)
    om = orc.model(GGUF(tinyllama_path))
    prompt = synth.prompt_ids(16, 32000, seed=0)
    st = m.state(max_ctx=64)
    st.enable_dump(True)
    om.reset()
    for pos in range(3):
        x = om.embed(int(prompt[pos]))
        ref_logits, ref_dump = om.forward(x, pos, dump=True)
        logits = st.forward_embedded(x, pos)
        dump = st.dump()
        for l in range(1, 23):
            assert rel_l2(dump[l], ref_dump[l]) < LAYER_TOL, (pos, l)
        assert rel_l2(logits, ref_logits) < LAYER_TOL
    cap = 32
    got, logits = st.generate_capped(prompt, cap, want_logits=True)
    ref, margins, ref_logits = oracle_greedy(orc, om, prompt, cap)
    agree = compare_tokens(got, ref, margins)
    if agree == cap:
        assert rel_l2(logits, ref_logits) < LAYER_TOL
    st.close()
    m.close()
