"""Batched sequences on the tensor-core path (tir_batch_*): every sequence of a
batch must decode what the oracle's generate_capped (src/lib.rs:239-314)
decodes for it alone -- greedy ids identical wherever the oracle's top-2 logit
margin exceeds 1e-3 -- both after a batched prefill and token by token."""
import numpy as np
import pytest

from tir import synth
from test_decode_gpu import compare_tokens, oracle_greedy

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(cuda, tirlib, orc, tiny_path):
    from oracle.gguf_ref import GGUF
    m = tirlib.Model(tiny_path)
    yield m, orc.model(GGUF(tiny_path))
    m.close()


# (2, 380, 12): decode positions 380-391 walk three shared-memory windows of
# earlier key/value rows in the decode attention (the last one staged after
# the kernel's dependency wait, with the new row read back from the cache)
@pytest.mark.parametrize("n_seqs,n_prompt,cap", [(3, 5, 10), (2, 40, 6), (1, 1, 4), (2, 380, 12)])
def test_batch_generate_matches_oracle_per_sequence(tirlib, orc, tiny, n_seqs, n_prompt, cap):
    m, om = tiny
    vocab = m.info["vocab"]
    prompts = np.stack([synth.prompt_ids(n_prompt, vocab, seed=100 + s) for s in range(n_seqs)])
    b = tirlib.Batch(m, n_seqs, max_ctx=n_prompt + cap + 1, max_tokens_per_seq=n_prompt)
    got = b.generate(prompts, cap)
    assert got.shape == (n_seqs, cap) and len(b) == n_prompt + cap
    for s in range(n_seqs):
        ref, margins, _ = oracle_greedy(orc, om, prompts[s], cap)
        compare_tokens(got[s], ref, margins)
    # deterministic, and the same as feeding the prompt one token at a time
    np.testing.assert_array_equal(b.generate(prompts, cap), got)
    b.reset()
    nxt = None
    for i in range(n_prompt):
        nxt = b.step(prompts[:, i:i + 1])
    steps = [nxt]
    for _ in range(cap - 1):
        steps.append(b.step(steps[-1][:, None]))
    by_token = np.stack(steps, axis=1)
    for s in range(n_seqs):
        ref, margins, _ = oracle_greedy(orc, om, prompts[s], cap)
        compare_tokens(by_token[s], ref, margins)
    b.close()


def test_batch_errors(tirlib, tiny):
    m, _ = tiny
    b = tirlib.Batch(m, 2, max_ctx=8, max_tokens_per_seq=4)
    with pytest.raises(tirlib.TirError) as e:
        b.step(np.ones((2, 5), np.int32))
    assert e.value.name == "INVALID_ARG"
    with pytest.raises(tirlib.TirError) as e:
        b.generate(np.ones((2, 4), np.int32), 5)
    assert e.value.name == "CTX_OVERFLOW"
    with pytest.raises(tirlib.TirError) as e:
        b.step(np.array([[1], [m.info["vocab"]]], np.int32))
    assert e.value.name == "BAD_TOKEN"
    assert len(b) == 0
    # the error is cleared with the reset: the batch decodes again
    nxt = b.step(np.array([[1], [2]], np.int32))
    assert nxt.shape == (2,) and len(b) == 1
    nxt = b.step(nxt[:, None])
    assert len(b) == 2
    b.close()


def _oracle_tokens(orc, om, ids, cap):
    """Greedy continuation of `ids` on the oracle, with top-2 margins."""
    return oracle_greedy(orc, om, np.asarray(ids, np.int32), cap)


def test_ragged_steps_match_each_sequence(tirlib, orc, tiny):
    """Sequences of different prompt lengths, fed in chunks and decoded in
    mixed steps (some prefilling, some decoding, some idle); every sequence
    must still decode what the oracle decodes for it alone."""
    m, om = tiny
    vocab = m.info["vocab"]
    prompts = [synth.prompt_ids(n, vocab, seed=300 + n) for n in (3, 17, 9)]
    b = tirlib.Batch(m, 3, max_ctx=64, max_tokens_per_seq=8)
    got = [[], [], []]
    fed = [0, 0, 0]
    pending = [None, None, None]
    for _ in range(14):
        chunk = []
        for s_ in range(3):
            if fed[s_] < len(prompts[s_]):
                n = min(8, len(prompts[s_]) - fed[s_], 1 + (s_ + fed[s_]) % 5)  # uneven prompt chunks
                chunk.append(prompts[s_][fed[s_]:fed[s_] + n])
                fed[s_] += n
            elif len(got[s_]) < 6 and pending[s_] is not None and (s_ != 2 or len(got[2]) < 3 or _ % 2 == 0):
                chunk.append([pending[s_]])  # decode (sequence 2 idles every other step late on)
                got[s_].append(pending[s_])
            else:
                chunk.append([])
        nxt = b.step_ragged(chunk)
        for s_ in range(3):
            if len(chunk[s_]) > 0:
                pending[s_] = int(nxt[s_])
    for s_ in range(3):
        assert b.seq_len(s_) == len(prompts[s_]) + len(got[s_])
        ref, margins, _ = _oracle_tokens(orc, om, prompts[s_], len(got[s_]))
        compare_tokens(np.array(got[s_], np.int32), ref, margins)
    b.close()


def test_continuous_batching_reuses_pages(tirlib, orc, tiny):
    """A finished sequence is reset and its slot starts a new prompt while the
    other keeps decoding; pages go back to the pool and are reused."""
    m, om = tiny
    vocab = m.info["vocab"]
    b = tirlib.Batch(m, 2, max_ctx=48, max_tokens_per_seq=16, n_pages=4)
    assert b.free_pages() == 4
    p0, p1, p2 = (synth.prompt_ids(n, vocab, seed=400 + n) for n in (14, 5, 7))
    nxt = b.step_ragged([p0, p1])
    out0, out1 = [int(nxt[0])], [int(nxt[1])]
    for _ in range(4):
        nxt = b.step_ragged([[out0[-1]], [out1[-1]]])
        out0.append(int(nxt[0]))
        out1.append(int(nxt[1]))
    assert 4 - b.free_pages() == 2 + 1  # 18 positions -> 2 pages, 9 -> 1 page
    b.reset_seq(1)
    assert b.free_pages() == 4 - 2 and b.seq_len(1) == 0
    nxt = b.step_ragged([[out0[-1]], p2])  # slot 1 restarts with a new prompt
    out0.append(int(nxt[0]))
    out2 = [int(nxt[1])]
    for _ in range(3):
        nxt = b.step_ragged([[out0[-1]], [out2[-1]]])
        out0.append(int(nxt[0]))
        out2.append(int(nxt[1]))
    for prompt, out in ((p0, out0), (p1, out1), (p2, out2)):
        ref, margins, _ = _oracle_tokens(orc, om, prompt, len(out))
        compare_tokens(np.array(out, np.int32), ref, margins)
    # one free page left: a step needing two more does not fit, and nothing changes
    assert b.free_pages() == 1
    with pytest.raises(tirlib.TirError) as e:
        b.step_ragged([synth.prompt_ids(16, vocab, seed=8), synth.prompt_ids(16, vocab, seed=9)])
    assert e.value.name == "OOM"
    assert b.seq_len(0) == len(p0) + len(out0) - 1 and b.seq_len(1) == len(p2) + len(out2) - 1
    assert b.free_pages() == 1
    b.close()


def test_batch_logits_match_each_sequence(tirlib, orc, small_path):
    """tir_batch_logits: every sequence's last-row logits after a prefill step
    and after a decode step agree with the oracle's forward of that sequence
    alone, and their argmax is the step's greedy id."""
    from oracle.gguf_ref import GGUF
    from test_decode_gpu import rel_l2
    m = tirlib.Model(small_path)
    vocab = m.info["vocab"]
    b = tirlib.Batch(m, 3, max_ctx=32, max_tokens_per_seq=8)
    prompts = np.stack([synth.prompt_ids(8, vocab, seed=700 + i) for i in range(3)])
    nxt = b.step(prompts)
    lg = b.logits()
    np.testing.assert_array_equal(np.argmax(lg[:, ::-1], axis=1) * -1 + vocab - 1, nxt)
    om = orc.model(GGUF(small_path))
    for i in range(3):
        om.reset()
        ref = None
        for pos, t in enumerate(prompts[i]):
            ref = om.forward(om.embed(int(t)), pos)
        assert rel_l2(lg[i], ref) < 1e-4
    nxt2 = b.step(nxt.reshape(3, 1))
    lg2 = b.logits()
    np.testing.assert_array_equal(np.argmax(lg2[:, ::-1], axis=1) * -1 + vocab - 1, nxt2)
    # sequence 0 decodes while 1 and 2 idle: its logits are its own, theirs zero
    nxt3 = b.step_ragged([[int(nxt2[0])], [], []])
    lg3 = b.logits()
    assert not lg3[1:].any()
    om.reset()
    for pos, t in enumerate(list(prompts[0]) + [int(nxt[0]), int(nxt2[0])]):
        ref = om.forward(om.embed(int(t)), pos)
    assert rel_l2(lg3[0], ref) < 1e-4
    assert int(nxt3[0]) == vocab - 1 - int(np.argmax(lg3[0][::-1]))
    b.close()
    m.close()
