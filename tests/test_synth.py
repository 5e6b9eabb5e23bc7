"""The synthetic-model writer: shapes, determinism, Q8_0 quantisation."""
import numpy as np

from tir import synth


def test_quantize_q8_0_roundtrip(orc):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((8, 128)) * 0.02).astype(np.float32)
    q = synth.quantize_q8_0(x)
    assert q.shape == (8, 128 // 32 * 34)
    deq = orc.q8_dequant(q.reshape(-1)).reshape(8, 128)
    scale = np.abs(x.reshape(8, 4, 32)).max(axis=2) / 127
    err = np.abs(deq - x).reshape(8, 4, 32).max(axis=2)
    assert np.all(err <= scale * 0.51 + np.abs(x.reshape(8, 4, 32)).max(axis=2) * 2e-3)


def test_tensor_specs_tinyllama():
    specs = {n: (d, s) for n, d, s in synth.tensor_specs(synth.PRESETS["tinyllama"])}
    assert specs["token_embd.weight"] == (8, [2048, 32000])
    assert specs["blk.21.attn_k.weight"] == (8, [2048, 256])
    assert specs["blk.0.ffn_down.weight"] == (8, [5632, 2048])
    assert specs["output.weight"] == (8, [2048, 32000])
    assert len(specs) == 3 + 22 * 9
    q8 = sum(np.prod(s) // 32 * 34 for _, (d, s) in specs.items() if d == 8)
    # weight bytes one decode step streams: 22 layers + lm_head (+ one embedding row)
    per_layer = sum(np.prod(specs[f"blk.0.{n}.weight"][1]) // 32 * 34
                    for n in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"))
    assert per_layer == 46_809_088 - 2 * 2048 * 4
    assert q8 == 22 * per_layer + 2 * 69_632_000


def test_prompt_ids_deterministic_and_in_range():
    a = synth.prompt_ids(64, 32000, seed=5)
    assert np.array_equal(a, synth.prompt_ids(64, 32000, seed=5))
    assert a.min() >= 3 and a.max() < 32000
    assert not np.array_equal(a, synth.prompt_ids(64, 32000, seed=6))


def test_gemv_case_layout():
    x, blocks = synth.gemv_case(64, 3, seed=1)
    assert x.shape == (64,) and blocks.shape == (3, 68)
    q = blocks.reshape(3, 2, 34)[:, :, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
