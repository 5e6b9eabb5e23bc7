"""Pins the CPU oracle against the reference's own known-answer unit tests
(tests/golden/reference_kat.json, extracted from src/math.rs, src/kernels.rs,
src/tokenizer.rs) and against independent restatements of the conversions it
depends on (the `half` crate's RNE f32->f16, Rust's `round`/`as i8`)."""
import numpy as np
import pytest


def q8_block(scale, weights):
    """src/math.rs:241-246 q8_block: f16 scale LE + 32 int8."""
    h = np.float16(scale).view(np.uint16)
    return bytes([int(h) & 0xff, int(h) >> 8]) + bytes(np.array(weights, np.int8).view(np.uint8))


def test_activated_q8_first_block(orc, kat):
    c = kat["activated_q8_first_block"]
    out = orc.activated_q8(np.full(c["input_len"], c["input_value"], np.float32))
    assert list(out[:34]) == c["expected_first_block"]


def test_dot_prod_f32(orc, kat):
    c = kat["dot_prod_f32"]
    assert orc.dot_prod_f32(c["a"], c["b"]) == c["expected"]


def test_q8_dequant_block(orc, kat):
    c = kat["q8_dequant_block"]
    raw = np.array(c["raw_block"], np.uint8)
    assert list(raw[2:].view(np.int8)) == c["quantized"]
    assert abs(orc.f16_to_f32(int(raw[0]) | int(raw[1]) << 8) - c["scale"]) < 1e-10
    out = orc.q8_dequant(raw)
    np.testing.assert_allclose(out, c["dequantized"], rtol=0, atol=c["tolerance"])
    # dequantisation is exact: f32(q) * f32(scale) with one rounding
    scale = np.float32(orc.f16_to_f32(int(raw[0]) | int(raw[1]) << 8))
    np.testing.assert_array_equal(out, raw[2:].view(np.int8).astype(np.float32) * scale)


def test_dot_prod_q8(orc, kat):
    c = kat["dot_prod_q8"]
    block = np.frombuffer(q8_block(c["scale"], c["weights"]), np.uint8)
    assert orc.dot_prod_q8(np.full(32, c["a_value"], np.float32), block) == c["expected"]


def test_q8_matmul(orc, kat):
    c = kat["q8_matmul"]
    w = {"w1": c["w1"], "w2": c["w2"]}
    b = np.frombuffer(b"".join(q8_block(s, w[name]) for s, name in c["blocks"]), np.uint8)
    a = np.array(c["a"], np.float32)
    dense = orc.q8_dequant(b).reshape(2, 64)
    expected = np.array([orc.dot_prod_f32(a, row) for row in dense], np.float32)
    np.testing.assert_allclose(orc.q8_matmul(a, b, 2), expected, rtol=0, atol=c["tolerance"])


def test_rmsnorm(orc, kat):
    c = kat["rmsnorm"]
    np.testing.assert_allclose(orc.rmsnorm(c["a"], c["w"]), c["expected"], rtol=0, atol=c["tolerance"])


def test_softmax(orc, kat):
    c = kat["softmax"]
    out = orc.softmax(c["x"])
    np.testing.assert_allclose(out, c["expected"], rtol=0, atol=c["tolerance"])
    assert abs(float(np.sum(out, dtype=np.float32)) - 1.0) < 1e-6


def test_rope(orc, kat):
    c = kat["rope"]
    theta = orc.rope_angles(c["base"], c["pos"], c["dim"])
    q, k = orc.rope(c["query"], c["key"], theta, c["dim"])
    np.testing.assert_allclose(q, c["expected"], rtol=0, atol=c["tolerance"])
    np.testing.assert_allclose(k, c["expected"], rtol=0, atol=c["tolerance"])


def test_sample(orc, kat):
    c = kat["sample"]
    assert orc.sample(c["logits"]) == c["expected"]


def test_sample_ties_go_to_last(orc):
    # Iterator::max_by returns the last of equal maxima (src/tokenizer.rs:160-165)
    assert orc.sample([1.0, 3.0, 3.0, 2.0]) == 2
    assert orc.sample([]) == 0
    # total_cmp: +0.0 > -0.0, NaN above +inf
    assert orc.sample([0.0, -0.0]) == 0
    assert orc.sample([np.inf, np.nan, 1.0]) == 1


def test_f16_rne_matches_numpy(orc):
    """`half` 2.7.1 f16::from_f32 is round-to-nearest-even, as numpy's cast."""
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504.0, 65520.0, 1e-8, 5.96e-8, 2.98e-8, 6.1e-5, np.inf, -np.inf], np.float32),
    ]).astype(np.float32)
    ours = np.array([orc.f32_to_f16(v) for v in vals], np.uint16)
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(ours, ref)
    back = np.array([orc.f16_to_f32(h) for h in ours], np.float32)
    np.testing.assert_array_equal(back, ours.view(np.float16).astype(np.float32))


def _activated_q8_py(x):
    """Loop restatement of src/kernels.rs:8-31 (round half away, saturating)."""
    x = np.asarray(x, np.float32)
    out = bytearray()
    for b in range(len(x) // 32):
        blk = x[32 * b:32 * b + 32]
        best = 0
        for i in range(1, 32):
            if not (abs(blk[best]) > abs(blk[i])):
                best = i
        scale = np.float32(blk[best]) / np.float32(127.0)
        out += np.array([scale], np.float16).tobytes()
        for v in blk:
            with np.errstate(all="ignore"):
                r = np.float32(v) / scale
            if np.isnan(r):
                q = 0
            else:
                q = int(np.floor(abs(r) + 0.5)) * (1 if r >= 0 else -1)
                q = max(-128, min(127, q))
            out.append(q & 0xff)
    return np.frombuffer(bytes(out), np.uint8)


@pytest.mark.parametrize("case", ["random", "negative_max", "ties", "zeros", "halves"])
def test_activated_q8_semantics(orc, case):
    rng = np.random.default_rng(7)
    if case == "random":
        x = rng.standard_normal(256).astype(np.float32) * 3
    elif case == "negative_max":
        x = rng.standard_normal(64).astype(np.float32)
        x[5], x[40] = -9.0, -7.5
    elif case == "ties":
        x = rng.standard_normal(64).astype(np.float32)
        x[3], x[9] = 4.0, -4.0      # last of equal |x| wins -> negative scale
        x[33], x[50] = -4.0, 4.0    # -> positive scale
    elif case == "zeros":
        x = np.zeros(64, np.float32)
    else:
        x = (np.arange(64, dtype=np.float32) - 31.5) * np.float32(0.5)
    np.testing.assert_array_equal(orc.activated_q8(x), _activated_q8_py(x))


def test_q8_act_matmul_integer_block_dot(orc):
    rng = np.random.default_rng(3)
    k, n = 256, 5
    xq = orc.activated_q8(rng.standard_normal(k).astype(np.float32))
    w = np.frombuffer(b"".join(q8_block(float(s), rng.integers(-127, 128, 32))
                               for s in rng.uniform(0.001, 0.01, n * k // 32)), np.uint8)
    out = orc.q8_act_matmul(xq, w, n)
    for r in range(n):
        total = np.float32(-0.0)
        row = w[r * (k // 32) * 34:(r + 1) * (k // 32) * 34]
        for b in range(k // 32):
            xa, wb = xq[34 * b:34 * b + 34], row[34 * b:34 * b + 34]
            isum = int(np.dot(xa[2:].view(np.int8).astype(np.int64), wb[2:].view(np.int8).astype(np.int64)))
            sa = np.float32(xa[:2].view(np.float16)[0])
            sb = np.float32(wb[:2].view(np.float16)[0])
            total = np.float32(total + np.float32(np.float32(np.float32(isum) * sa) * sb))
        assert out[r] == total


def test_fast_mode_is_bit_identical(orc, small_path):
    """The tests run the oracle in its fast mode (eight matrix rows per pass,
    attention heads in parallel); every row and head keeps the reference's
    operation order, so its forward must equal the reference-order forward bit
    for bit, including a q8_matmul whose row count is not a multiple of 8."""
    from oracle.gguf_ref import GGUF
    from tir import synth
    x, blocks = synth.gemv_case(1024, 203, seed=4)
    outs = {}
    for fast in (False, True):
        orc.set_fast(fast)
        om = orc.model(GGUF(small_path))
        steps = [om.forward(om.embed(t), p, dump=True) for p, t in enumerate([3, 77, 1500, 9])]
        outs[fast] = (steps, orc.q8_matmul(x, blocks.reshape(-1), 203))
    orc.set_fast(True)
    for (la, da), (lb, db) in zip(outs[False][0], outs[True][0]):
        np.testing.assert_array_equal(la, lb)
        np.testing.assert_array_equal(da, db)
    np.testing.assert_array_equal(outs[False][1], outs[True][1])
