"""Parity at the benchmarked workloads' own shapes: the TinyLlama-shape model
(22 layers, hidden 2048, 32/4 heads, FFN 5632, vocab 32000) through the C ABI
against the oracle's restatement of the reference's forward
(src/forward.rs:13-258) and decode driver (src/lib.rs:239-314), on the same
synthetic GGUF and the same seeded token ids as bench.py:

* batch-1 decode, 16 prompt ids + 128 greedy steps: all 144 forwards;
* long context, 1792 prompt ids + 256 greedy steps up to context 2048 (the
  attention phase then splits each KV head over up to 37 CTAs and the last
  split merges them);
* 64 sequences x (128 prompt ids + 128 greedy steps) through tir_batch;
* 16 sequences x 512 prompt ids prefilled in one tir_batch step (8192 rows
  per tensor-core matmul).

Bars: per-layer hidden states within fp32 relative-L2 1e-4; greedy ids
identical wherever the oracle's top-2 logit margin exceeds 1e-3 (at the first
disagreement the margin must be <= 1e-3, and later ids are not compared).
"""
import numpy as np
import pytest

from tir import synth
from test_decode_gpu import LAYER_TOL, compare_tokens, oracle_greedy, rel_l2

pytestmark = pytest.mark.gpu

VOCAB = 32000


@pytest.fixture(scope="module")
def tl(cuda, tirlib, orc, tinyllama_path):
    from oracle.gguf_ref import GGUF
    m = tirlib.Model(tinyllama_path)
    yield m, orc.model(GGUF(tinyllama_path))
    m.close()


def oracle_trajectory(orc, om, prompt, cap, dump_at=()):
    """generate_capped on the oracle: the ids of every position (prompt, then
    greedy), the top-2 margin of each greedy step, the per-layer states of the
    positions in dump_at and the last forward's logits."""
    om.reset()
    ids = [int(t) for t in prompt]
    margins, dumps, logits = [], {}, None
    for pos in range(len(prompt) + cap):
        if pos >= len(prompt):
            srt = np.sort(logits)
            margins.append(float(srt[-1]) - float(srt[-2]))
            ids.append(orc.sample(logits))
        if pos in dump_at:
            logits, d = om.forward(om.embed(ids[pos]), pos, dump=True)
            dumps[pos] = d.copy()
        else:
            logits = om.forward(om.embed(ids[pos]), pos)
    return np.array(ids, np.int32), margins, dumps, logits


def check_layers(dump, ref, where):
    for l in range(1, ref.shape[0]):
        r = rel_l2(dump[l], ref[l])
        assert r < LAYER_TOL, (where, l, r)


def test_decode_16_plus_128(tl, orc):
    """The batch-1 benchmark workload in full: 16 prompt ids, 128 greedy ids."""
    m, om = tl
    prompt = synth.prompt_ids(16, VOCAB, seed=0)
    check_at = (0, 15, 64, 143)
    ids, margins, dumps, ref_logits = oracle_trajectory(orc, om, prompt, 128, check_at)
    st = m.state(max_ctx=160)
    got, logits = st.generate_capped(prompt, 128, want_logits=True)
    agree = compare_tokens(got, ids[16:], margins)
    if agree == 128:
        assert rel_l2(logits, ref_logits) < LAYER_TOL
    # per-layer states along the oracle's trajectory (its ids fed back)
    st.reset()
    st.enable_dump(True)
    for pos in range(144):
        st.forward(int(ids[pos]), pos)
        if pos in check_at:
            check_layers(st.dump(), dumps[pos], pos)
    st.close()


def test_long_context_1792_plus_256(tl, orc):
    """Context 2048: the attention splits reach 37 per KV head, merged by the
    last split to finish."""
    m, om = tl
    prompt = synth.prompt_ids(1792, VOCAB, seed=2)
    check_at = (1791, 2047)
    ids, margins, dumps, ref_logits = oracle_trajectory(orc, om, prompt, 256, check_at)
    st = m.state(max_ctx=2048)
    got, logits = st.generate_capped(prompt, 256, want_logits=True)
    agree = compare_tokens(got, ids[1792:], margins)
    if agree == 256:
        assert rel_l2(logits, ref_logits) < LAYER_TOL
    st.reset()
    st.enable_dump(True)
    st.prefill(ids[:1791], want_logits=False)
    st.forward(int(ids[1791]), 1791)
    check_layers(st.dump(), dumps[1791], 1791)
    for pos in range(1792, 2048):
        st.forward(int(ids[pos]), pos)
    check_layers(st.dump(), dumps[2047], 2047)
    st.close()


def test_batched_64_sequences(tl, tirlib, orc):
    """64 sequences x (128 prompt + 128 greedy) in one batch; four of them
    (first, last and two between) against the oracle run alone."""
    m, om = tl
    n_seqs, n_prompt, cap = 64, 128, 128
    prompts = np.stack([synth.prompt_ids(n_prompt, VOCAB, seed=1000 + s) for s in range(n_seqs)])
    b = tirlib.Batch(m, n_seqs, max_ctx=n_prompt + cap, max_tokens_per_seq=n_prompt)
    got = b.generate(prompts, cap)
    b.close()
    for s in (0, 21, 42, 63):
        ref, margins, _ = oracle_greedy(orc, om, prompts[s], cap)
        compare_tokens(got[s], ref, margins)


def test_prefill_16x512(tl, tirlib, orc):
    """16 x 512 prompt ids in one step: the last-row logits and next ids of
    two sequences, and the per-layer states of three rows, against the
    oracle's token-by-token prefill."""
    m, om = tl
    n_seqs, n = 16, 512
    prompts = np.stack([synth.prompt_ids(n, VOCAB, seed=500 + s) for s in range(n_seqs)])
    b = tirlib.Batch(m, n_seqs, max_ctx=n, max_tokens_per_seq=n)
    rows = [100, n - 1, 7 * n + n - 1]  # seq 0 pos 100, seq 0 last, seq 7 last
    b.dump_rows(rows)
    nxt = b.step(prompts)
    logits = b.logits()
    dump = b.dump()
    b.close()
    for k, s in enumerate((0, 7)):
        om.reset()
        for pos in range(n):
            want = pos in (100, n - 1) if s == 0 else pos == n - 1
            if want:
                lg, d = om.forward(om.embed(int(prompts[s, pos])), pos, dump=True)
                row = s * n + pos
                check_layers(np.concatenate([d[:1], dump[rows.index(row)]]), d, (s, pos))
            else:
                lg = om.forward(om.embed(int(prompts[s, pos])), pos)
        assert rel_l2(logits[s], lg) < LAYER_TOL, s
        srt = np.sort(lg)
        if nxt[s] != orc.sample(lg):
            assert srt[-1] - srt[-2] <= 1e-3, s
