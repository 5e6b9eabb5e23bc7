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
matmul it feeds by ~1e-4 of its norm; later layers quantise again, so one
flip cascades.  test_qact_flips_counted_and_layers_tight_without_them counts
the flips and holds every layer upstream of the first one to 1e-4."""
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


def _int8(blocks):
    b = np.asarray(blocks, np.uint8).reshape(-1, 34)
    return b[:, 2:].copy().view(np.int8).astype(np.int32)


def _f32_tensor(gguf, name):
    return np.frombuffer(gguf.tensor_bytes(name).tobytes(), np.float32)


@pytest.mark.parametrize("preset", ["tiny", "small"])
def test_qact_flips_counted_and_layers_tight_without_them(cuda, tirlib, orc, tiny_path, small_path, preset):
    """The looser bound above rests on int8 rounding flips; this counts them.
    The fused kernel's own activated_q8 blocks (tir_debug_dump_qact) are
    compared (1) with activated_q8 of the same input recomputed on the host
    from the kernel's own hidden state (rmsnorm summed in another order can
    move an ulp, so a flip there is one step of a value at a rounding edge,
    and rare), and (2) with the oracle's blocks on its own trajectory, for the
    q|k|v, o and lm_head inputs.  Every layer with no flip in its own or any
    earlier quantised input must then hold the Normal-mode bar, 1e-4."""
    from oracle.gguf_ref import GGUF
    path = tiny_path if preset == "tiny" else small_path
    gg = GGUF(path)
    m = tirlib.Model(path)
    m.set_mode(1)
    om = orc.model(gg, mode=1)
    L = m.info["layers"]
    attn_w = [_f32_tensor(gg, f"blk.{l}.attn_norm.weight") for l in range(L)]
    out_w = _f32_tensor(gg, "output_norm.weight")
    st = m.state(max_ctx=64)
    st.enable_dump(True)
    om.reset()
    same_flips, traj_flips, tight = 0, 0, 0
    for pos, t in enumerate(synth.prompt_ids(6, m.info["vocab"], seed=3)):
        x = om.embed(int(t))
        ref_logits, ref_dump, ref_attn = om.forward_attn(x, pos)
        logits = st.forward_embedded(x, pos)
        dump, q = st.dump(), st.dump_qact()
        flipped = False
        for l in range(L):
            got = _int8(q[2 * l])
            same = _int8(orc.activated_q8(orc.rmsnorm(dump[l], attn_w[l])))
            d = np.abs(got - same)
            assert d.max() <= 1 and (d > 0).sum() <= max(2, got.size // 1000), (pos, l, int((d > 0).sum()))
            same_flips += int((d > 0).sum())
            n = int((got != _int8(orc.activated_q8(orc.rmsnorm(ref_dump[l], attn_w[l])))).sum())
            n += int((_int8(q[2 * l + 1]) != _int8(orc.activated_q8(ref_attn[l]))).sum())
            traj_flips += n
            flipped |= n > 0
            r = rel_l2(dump[l + 1], ref_dump[l + 1])
            if flipped:
                assert r < QACT_LAYER_TOL, (pos, l, r)
            else:
                assert r < 1e-4, (pos, l, r)
                tight += 1
        flipped |= bool((_int8(q[2 * L]) != _int8(orc.activated_q8(orc.rmsnorm(ref_dump[L], out_w)))).any())
        assert rel_l2(logits, ref_logits) < (QACT_LAYER_TOL if flipped else 1e-4)
    print(f"{preset}: {same_flips} same-input flips, {traj_flips} trajectory flips, {tight} of {6 * L} layers at 1e-4")
    assert tight > 0
    st.close()
    m.close()
