"""Mode::Quantize (src/data.rs:16-20, src/forward.rs:261-275) in the fused decode
kernel: the q, k, v, o and lm_head matmuls quantise their input with
activated_q8 (src/kernels.rs:8-31) and take integer block dots
(dot_prod_act_q8, src/math.rs:39-50); the FFN stays on q8_matmul.  Checked
against the oracle's Mode::Quantize forward on the same weights and ids:
greedy ids identical wherever the oracle's top-2 margin exceeds 1e-3 (the bar
of the Normal-mode tests), and per-layer hidden states within relative-L2
QACT_LAYER_TOL.  That bound is looser than Normal mode's 1e-4 on purpose: the
int8 rounding round(x / scale) turns an ulp-level difference in its input
(an rmsnorm sum or an attention output accumulated in another order) into a
whole quantisation step now and then, and one step moves every output of the
matmul it feeds by ~1e-4 of its norm; later layers quantise again.  Where no
step flips, the hidden states match to ~1e-7."""
import numpy as np
import pytest

from tir import synth
from test_decode_gpu import compare_tokens, oracle_greedy, rel_l2

pytestmark = pytest.mark.gpu

QACT_LAYER_TOL = 2e-2


@pytest.fixture(scope="module")
def qmodels(cuda, tirlib, orc, tiny_path, small_path):
    from oracle.gguf_ref import GGUF
    out = {}
    for name, path in (("tiny", tiny_path), ("small", small_path)):
        m = tirlib.Model(path)
        m.set_mode(1)
        out[name] = (m, orc.model(GGUF(path), mode=1))
    yield out
    for m, _ in out.values():
        m.close()


@pytest.mark.parametrize("name", ["tiny", "small"])
def test_qact_per_layer_hidden_states(qmodels, name):
    m, om = qmodels[name]
    st = m.state(max_ctx=64)
    st.enable_dump(True)
    om.reset()
    for pos, t in enumerate(synth.prompt_ids(6, m.info["vocab"], seed=3)):
        x = om.embed(int(t))
        ref_logits, ref_dump = om.forward(x, pos, dump=True)
        logits = st.forward_embedded(x, pos)
        dump = st.dump()
        for l in range(1, dump.shape[0]):
            assert rel_l2(dump[l], ref_dump[l]) < QACT_LAYER_TOL, (pos, l, rel_l2(dump[l], ref_dump[l]))
        assert rel_l2(logits, ref_logits) < QACT_LAYER_TOL
    st.close()


@pytest.mark.parametrize("name,n_prompt,cap", [("tiny", 8, 24), ("small", 12, 40)])
def test_qact_generate_capped_tokens(qmodels, orc, name, n_prompt, cap):
    m, om = qmodels[name]
    prompt = synth.prompt_ids(n_prompt, m.info["vocab"], seed=n_prompt + 100)
    st = m.state(max_ctx=n_prompt + cap)
    got, logits = st.generate_capped(prompt, cap, want_logits=True)
    ref, margins, ref_logits = oracle_greedy(orc, om, prompt, cap)
    if compare_tokens(got, ref, margins) == cap:
        assert rel_l2(logits, ref_logits) < QACT_LAYER_TOL
    st.close()


def test_mode_switch_on_a_live_state(tirlib, orc, small_path):
    """A state follows the model's mode from its next launch on; switching back
    reproduces the Normal-mode bits."""
    from oracle.gguf_ref import GGUF
    m = tirlib.Model(small_path)
    prompt = synth.prompt_ids(8, m.info["vocab"], seed=5)
    st = m.state(max_ctx=32)
    normal = st.generate_capped(prompt, 12)
    m.set_mode(1)
    quant = st.generate_capped(prompt, 12)
    ref, margins, _ = oracle_greedy(orc, orc.model(GGUF(small_path), mode=1), prompt, 12)
    compare_tokens(quant, ref, margins)
    m.set_mode(0)
    np.testing.assert_array_equal(st.generate_capped(prompt, 12), normal)
    with pytest.raises(tirlib.TirError) as e:
        m.set_mode(2)
    assert e.value.name == "INVALID_ARG"
    st.close()
    m.close()
