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


@pytest.mark.parametrize("n_seqs,n_prompt,cap", [(3, 5, 10), (2, 40, 6), (1, 1, 4)])
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
