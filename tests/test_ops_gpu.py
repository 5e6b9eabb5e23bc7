"""Op-level parity on the GPU: each tir_* kernel (through the C ABI) against the
CPU oracle on the same seeded inputs.  Bit-exact where the reference's
arithmetic is exact (dequantisation, embedding, activation quantisation,
integer block dots, RoPE, argmax); f32 tolerances written per test otherwise."""
import numpy as np
import pytest

from tir import synth

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.array(a, copy=True)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def split_layout(torch, tirlib, blocks, rows, k):
    b = dev(torch, np.ascontiguousarray(blocks, np.uint8).reshape(-1))
    q = torch.empty(rows * k, dtype=torch.uint8, device="cuda")
    s = torch.empty(rows * tirlib.q8_scale_stride(k), dtype=torch.int16, device="cuda")
    tirlib.q8_repack(b, rows, k, q, s)
    return q, s


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_repack_layout(cuda, tirlib):
    torch = cuda
    x, blocks = synth.gemv_case(1408, 6, seed=2)
    q, s = split_layout(torch, tirlib, blocks, 6, 1408)
    b = blocks.reshape(6, 44, 34)
    np.testing.assert_array_equal(host(q).reshape(6, 1408), b[:, :, 2:].reshape(6, 1408))
    sk = tirlib.q8_scale_stride(1408)
    sc = host(s).view(np.uint16).reshape(6, sk)
    np.testing.assert_array_equal(sc[:, :44], b[:, :, :2].copy().view(np.uint16).reshape(6, 44))
    assert np.all(sc[:, 44:] == 0)


# (K, N): the GEMV sweep shapes (q/o, k/v, gate/up, down, lm_head) plus ragged ones
SHAPES = [(2048, 2048), (2048, 256), (2048, 5632), (5632, 2048), (2048, 32000), (1408, 100), (96, 7),
          (64, 2), (6144, 40), (512, 1)]


@pytest.mark.parametrize("k,n", SHAPES)
def test_q8_matmul_vs_oracle(cuda, tirlib, orc, k, n):
    torch = cuda
    x, blocks = synth.gemv_case(k, n, seed=k + n)
    ref = orc.q8_matmul(x, blocks.reshape(-1), n)
    q, s = split_layout(torch, tirlib, blocks, n, k)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    tirlib.q8_matmul(dev(torch, x), q, s, out, n, k)
    got = host(out)
    # f32 with a different summation order: rel-L2 bound 1e-5 (observed ~1e-7)
    assert rel_l2(got, ref) < 1e-5
    scale = np.abs(x).sum() * 127 * np.abs(blocks.reshape(n, -1, 34)[:, :, :2].copy().view(np.float16)).max()
    assert np.max(np.abs(got - ref)) < 1e-5 * scale + 1e-30


def tiled_layout(torch, tirlib, blocks, rows, k):
    w = torch.empty(tirlib.q8_tiled_bytes(rows, k), dtype=torch.uint8, device="cuda")
    tirlib.q8_repack_tiled(dev(torch, np.ascontiguousarray(blocks, np.uint8).reshape(-1)), rows, k, w)
    return w


def test_repack_tiled_layout(cuda, tirlib):
    """Warp-sliced tile-major layout: tiles of R rows (last one zero-padded);
    in a tile, the slice of (row lane rl, column warp wi) -- rows rl + RL j
    (j < 2), blocks [32 wi, 32 wi + nbw) -- is one chunk: quants, then f16
    scales (nbw rounded up to 8 per row), chunks in (rl, wi) order."""
    torch = cuda
    for rows, k in [(29, 1408), (5, 5632), (7, 96)]:
        _, blocks = synth.gemv_case(k, rows, seed=5)
        w = host(tiled_layout(torch, tirlib, blocks, rows, k))
        nb = k // 32
        wpr = (nb + 31) // 32
        RL = 12 // wpr
        R = tirlib.q8_tile_rows(k)
        assert R == 2 * RL
        nbws = [min(32, nb - 32 * wi) for wi in range(wpr)]
        slice_bytes = [2 * (b * 32 + (b + 7) // 8 * 8 * 2) for b in nbws]
        lane_bytes = sum(slice_bytes)
        tile_bytes = RL * lane_bytes
        n_tiles = -(-rows // R)
        assert w.size == n_tiles * tile_bytes
        b = blocks.reshape(rows, nb, 34)
        seen = np.zeros(w.size, bool)
        for r in range(rows):
            t, rr = divmod(r, R)
            j, rl = divmod(rr, RL)
            for blk in range(nb):
                wi, bl = divmod(blk, 32)
                nbw = nbws[wi]
                base = t * tile_bytes + rl * lane_bytes + sum(slice_bytes[:wi])
                q = base + (j * nbw + bl) * 32
                sc = base + 2 * nbw * 32 + (j * ((nbw + 7) // 8 * 8) + bl) * 2
                np.testing.assert_array_equal(w[q:q + 32], b[r, blk, 2:])
                np.testing.assert_array_equal(w[sc:sc + 2], b[r, blk, :2])
                seen[q:q + 32] = True
                seen[sc:sc + 2] = True
        assert np.all(w[~seen] == 0)  # scale padding and padded rows


@pytest.mark.parametrize("k,n", [(2048, 2048), (2048, 256), (5632, 2048), (2048, 32000), (1408, 100), (96, 7),
                                 (6144, 40), (512, 1)])
def test_q8_matmul_tiled_vs_oracle(cuda, tirlib, orc, k, n):
    torch = cuda
    x, blocks = synth.gemv_case(k, n, seed=k + n)
    ref = orc.q8_matmul(x, blocks.reshape(-1), n)
    w = tiled_layout(torch, tirlib, blocks, n, k)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    tirlib.q8_matmul_tiled(dev(torch, x), w, out, n, k)
    got = host(out)
    assert rel_l2(got, ref) < 1e-5
    scale = np.abs(x).sum() * 127 * np.abs(blocks.reshape(n, -1, 34)[:, :, :2].copy().view(np.float16)).max()
    assert np.max(np.abs(got - ref)) < 1e-5 * scale + 1e-30


def test_q8_matmul_rejects_rows_longer_than_the_kernel_stages(cuda, tirlib):
    torch = cuda
    out = torch.empty(4, dtype=torch.float32, device="cuda")
    with pytest.raises(tirlib.TirError) as e:
        tirlib.q8_matmul(out, out, out, out, 4, 6144 + 32)
    assert e.value.name == "UNSUPPORTED_SHAPE"


def test_q8_matmul_reference_kat(cuda, tirlib, kat):
    """src/math.rs:359-379 on the GPU."""
    torch = cuda
    c = kat["q8_matmul"]
    from test_oracle_kat import q8_block
    w = {"w1": c["w1"], "w2": c["w2"]}
    blocks = np.frombuffer(b"".join(q8_block(sc, w[name]) for sc, name in c["blocks"]), np.uint8)
    a = np.array(c["a"], np.float32)
    dense = np.array([[np.float32(sc) * np.float32(v) for v in w[name]] for sc, name in c["blocks"]],
                     np.float32).reshape(2, 64)
    expected = dense.astype(np.float64) @ a.astype(np.float64)
    q, s = split_layout(torch, tirlib, blocks, 2, 64)
    out = torch.empty(2, dtype=torch.float32, device="cuda")
    tirlib.q8_matmul(dev(torch, a), q, s, out, 2, 64)
    np.testing.assert_allclose(host(out), expected, rtol=0, atol=c["tolerance"])


def test_q8_dequant_bit_exact(cuda, tirlib, orc, kat):
    torch = cuda
    _, blocks = synth.gemv_case(4096, 8, seed=9)
    flat = np.concatenate([np.array(kat["q8_dequant_block"]["raw_block"], np.uint8), blocks.reshape(-1)])
    nb = flat.size // 34
    out = torch.empty(nb * 32, dtype=torch.float32, device="cuda")
    tirlib.q8_dequant(dev(torch, flat), nb, out)
    np.testing.assert_array_equal(host(out), orc.q8_dequant(flat))


def test_embed_bit_exact(cuda, tirlib, orc):
    torch = cuda
    _, table = synth.gemv_case(2048, 50, seed=4)
    t = dev(torch, table.reshape(-1))
    out = torch.empty(2048, dtype=torch.float32, device="cuda")
    for i in (0, 17, 49):
        tirlib.embed(t, 50, i, 2048, out)
        np.testing.assert_array_equal(host(out), orc.embed(i, table.reshape(-1), 2048))
    with pytest.raises(tirlib.TirError) as e:
        tirlib.embed(t, 50, 50, 2048, out)
    assert e.value.name == "BAD_TOKEN"


@pytest.mark.parametrize("n", [3, 2048, 5632, 100000])
def test_rmsnorm(cuda, tirlib, orc, kat, n):
    torch = cuda
    rng = np.random.default_rng(n)
    if n == 3:
        x, w = np.array(kat["rmsnorm"]["a"], np.float32), np.array(kat["rmsnorm"]["w"], np.float32)
    else:
        x = rng.standard_normal(n).astype(np.float32) * 3
        w = (1 + rng.standard_normal(n) * 0.01).astype(np.float32)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    tirlib.rmsnorm(dev(torch, x), dev(torch, w), out, n)
    got = host(out)
    # The oracle's Sigma x^2 is a sequential f32 fold (relative drift ~ sqrt(n) ulp);
    # the kernel reduces in a tree.  Against float64 the kernel is within 2e-6.
    x64 = x.astype(np.float64)
    exact = x64 * w / np.sqrt(np.mean(x64 * x64) + 1e-5)
    np.testing.assert_allclose(got, exact, rtol=2e-6, atol=0)
    np.testing.assert_allclose(got, orc.rmsnorm(x, w), rtol=max(2e-6, 4 * np.sqrt(n) * 2.0 ** -24), atol=0)
    if n == 3:
        np.testing.assert_allclose(got, kat["rmsnorm"]["expected"], rtol=0, atol=kat["rmsnorm"]["tolerance"])


@pytest.mark.parametrize("n", [6, 145, 2048, 32000])
def test_softmax(cuda, tirlib, orc, kat, n):
    torch = cuda
    x = np.array(kat["softmax"]["x"], np.float32) if n == 6 else \
        (np.random.default_rng(n).standard_normal(n) * 4).astype(np.float32)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    tirlib.softmax(dev(torch, x), out, n)
    got = host(out)
    # the oracle's total is a sequential f32 fold (drift ~ sqrt(n) ulp); the
    # kernel's is a tree.  Against float64 the kernel is within 2e-6.
    x64 = x.astype(np.float64)
    e = np.exp(x64 - x64.max())
    np.testing.assert_allclose(got, e / e.sum(), rtol=2e-6, atol=1e-12)
    np.testing.assert_allclose(got, orc.softmax(x), rtol=max(2e-6, 4 * np.sqrt(n) * 2.0 ** -24), atol=1e-12)
    assert abs(float(got.astype(np.float64).sum()) - 1.0) < 1e-5
    if n == 6:
        np.testing.assert_allclose(got, kat["softmax"]["expected"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("pos", [0, 1, 7, 143, 2047])
def test_rope_bit_exact(cuda, tirlib, orc, pos):
    torch = cuda
    rng = np.random.default_rng(pos)
    q = rng.standard_normal(2048).astype(np.float32)
    k = rng.standard_normal(256).astype(np.float32)
    theta = orc.rope_angles(10000.0, pos, 64)
    rq, rk = orc.rope(q, k, theta, 64)
    dq, dk = dev(torch, q), dev(torch, k)
    tirlib.rope(dq, 2048, dk, 256, theta, 64)
    np.testing.assert_array_equal(host(dq), rq)
    np.testing.assert_array_equal(host(dk), rk)


def test_rope_reference_kat(cuda, tirlib, kat):
    torch = cuda
    c = kat["rope"]
    theta = tirlib.rope_angles(c["base"], c["pos"], c["dim"])
    dq, dk = dev(torch, np.array(c["query"], np.float32)), dev(torch, np.array(c["key"], np.float32))
    tirlib.rope(dq, 4, dk, 4, theta, c["dim"])
    np.testing.assert_allclose(host(dq), c["expected"], rtol=0, atol=c["tolerance"])
    np.testing.assert_allclose(host(dk), c["expected"], rtol=0, atol=c["tolerance"])


@pytest.mark.parametrize("case", ["kat", "random", "ties", "zeros", "big"])
def test_activated_q8_bit_exact(cuda, tirlib, orc, kat, case):
    torch = cuda
    rng = np.random.default_rng(11)
    if case == "kat":
        x = np.full(2048, kat["activated_q8_first_block"]["input_value"], np.float32)
    elif case == "random":
        x = (rng.standard_normal(2048) * 2).astype(np.float32)
    elif case == "ties":
        x = rng.standard_normal(128).astype(np.float32)
        x[3], x[9], x[40], x[41] = 4.0, -4.0, -2.0, 2.0
    elif case == "zeros":
        x = np.zeros(64, np.float32)
    else:
        x = (rng.standard_normal(5632) * 1e4).astype(np.float32)
    out = torch.zeros(x.size // 32 * 34, dtype=torch.uint8, device="cuda")
    tirlib.activated_q8(dev(torch, x), x.size, out)
    got = host(out)
    np.testing.assert_array_equal(got, orc.activated_q8(x))
    if case == "kat":
        assert list(got[:34]) == kat["activated_q8_first_block"]["expected_first_block"]


@pytest.mark.parametrize("k,n", [(2048, 2048), (2048, 256), (5632, 64), (64, 3)])
def test_q8_act_matmul_bit_exact(cuda, tirlib, orc, k, n):
    torch = cuda
    x, blocks = synth.gemv_case(k, n, seed=3 * k + n)
    xq = orc.activated_q8(x)
    q, s = split_layout(torch, tirlib, blocks, n, k)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    tirlib.q8_act_matmul(dev(torch, xq), q, s, out, n, k)
    np.testing.assert_array_equal(host(out), orc.q8_act_matmul(xq, blocks.reshape(-1), n))


@pytest.mark.parametrize("k,n,case", [(2048, 2048, "random"), (1024, 1536, "random"), (512, 768, "random"),
                                      (5632, 64, "random"), (2048, 300, "ties"), (1024, 96, "zeros")])
def test_q8_matmul_qact_vs_oracle(cuda, tirlib, orc, k, n, case):
    """The fused kernel's Mode::Quantize input staging and integer block dot
    (single-phase launch) against activated_q8 + q8_act_matmul: the same
    per-block terms, summed in another order (rel-L2 below 1e-6)."""
    torch = cuda
    x, blocks = synth.gemv_case(k, n, seed=7 * k + n)
    if case == "ties":  # equal |x| of opposite signs: the last one sets the scale's sign
        x[3], x[9], x[40], x[41] = 4.0, -4.0, -2.0, 2.0
    elif case == "zeros":
        x[:64] = 0.0
    q, s = split_layout(torch, tirlib, blocks, n, k)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    tirlib.q8_matmul_qact(dev(torch, x), q, s, out, n, k)
    ref = orc.q8_act_matmul(orc.activated_q8(x), blocks.reshape(-1), n)
    assert rel_l2(host(out), ref) < 1e-6


@pytest.mark.parametrize("case", ["random", "ties", "nan", "zeros", "empty", "big"])
def test_argmax_matches_sample(cuda, tirlib, orc, case):
    torch = cuda
    rng = np.random.default_rng(5)
    x = {"random": rng.standard_normal(32000).astype(np.float32),
         "ties": np.array([1, 5, 3, 5, 2, 5, 0], np.float32),
         "nan": np.array([1.0, np.inf, np.nan, 2.0], np.float32),
         "zeros": np.array([-0.0, 0.0, -0.0], np.float32),
         "empty": np.zeros(0, np.float32),
         "big": rng.standard_normal(1 << 20).astype(np.float32)}[case]
    out = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    xd = dev(torch, x) if x.size else torch.zeros(1, dtype=torch.float32, device="cuda")
    tirlib.argmax(xd, x.size, out)
    assert int(host(out)[0]) == orc.sample(x)


def _attention_ref(q, kc, vc, qh, kvh, n_ctx):
    """src/forward.rs:86-174 in float64: per head softmax(q.k/8) . v."""
    out = np.zeros(qh * 64)
    group = qh // kvh
    for h in range(qh):
        g = h // group
        K = kc[g, :n_ctx].astype(np.float64)
        V = vc[g, :n_ctx].astype(np.float64)
        s = K @ q[h * 64:(h + 1) * 64].astype(np.float64) / 8.0
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * 64:(h + 1) * 64] = p @ V
    return out


@pytest.mark.parametrize("n_ctx", [1, 33, 144, 2048])
def test_attention(cuda, tirlib, n_ctx):
    torch = cuda
    rng = np.random.default_rng(n_ctx)
    qh, kvh, max_ctx = 32, 4, 2048
    q = rng.standard_normal(qh * 64).astype(np.float32)
    kc = rng.standard_normal((kvh, max_ctx, 64)).astype(np.float32)
    vc = rng.standard_normal((kvh, max_ctx, 64)).astype(np.float32)
    out = torch.empty(qh * 64, dtype=torch.float32, device="cuda")
    tirlib.attention(dev(torch, q), dev(torch, kc), dev(torch, vc), out, qh, kvh, 64, n_ctx, max_ctx)
    assert rel_l2(host(out), _attention_ref(q, kc, vc, qh, kvh, n_ctx)) < 1e-5


def test_swiglu(cuda, tirlib, orc):
    torch = cuda
    k, f = 2048, 5632
    rng = np.random.default_rng(21)
    x = rng.standard_normal(k).astype(np.float32)
    _, wg = synth.gemv_case(k, f, seed=1)
    _, wu = synth.gemv_case(k, f, seed=2)
    _, wd = synth.gemv_case(f, k, seed=3)
    ref = orc.swiglu(x, wg.reshape(-1), wu.reshape(-1), wd.reshape(-1), f)
    g = split_layout(torch, tirlib, wg, f, k)
    u = split_layout(torch, tirlib, wu, f, k)
    d = split_layout(torch, tirlib, wd, k, f)
    out = torch.empty(k, dtype=torch.float32, device="cuda")
    tirlib.swiglu(dev(torch, x), g, u, d, out, k, f)
    assert rel_l2(host(out), ref) < 1e-5


@pytest.mark.parametrize("tokens,k,n", [(64, 2048, 2560), (300, 2048, 2048), (128, 5632, 2048), (7, 128, 7),
                                        (1, 2048, 32000), (257, 1024, 130), (64, 2048, 11264), (33, 5632, 2048)])
def test_q8_matmul_batch_vs_oracle(cuda, tirlib, orc, tokens, k, n):
    """Tensor-core batched matmul (3-pass f16 split, f32 accumulation): every
    token row against the float64 product of the dequantised weights, and
    three rows against the oracle's q8_matmul; rel-L2 below 1e-5 per row."""
    torch = cuda
    rng = np.random.default_rng(tokens + k + n)
    _, blocks = synth.gemv_case(k, n, seed=k * 3 + n)
    x = rng.standard_normal((tokens, k)).astype(np.float32)
    x[0, :] *= 1e-3  # a token of much smaller magnitude: per-token scaling
    w = tirlib.q8_gemm_prepare(dev(torch, blocks.reshape(-1)), n, k)
    y = torch.empty(tokens * n, dtype=torch.float32, device="cuda")
    tirlib.q8_matmul_batch(dev(torch, x), tokens, w, y, n, k)
    got = host(y).reshape(tokens, n)
    bl = blocks.reshape(n, k // 32, 34)
    scale = bl[..., :2].copy().view(np.float16).astype(np.float64)      # [n, k/32, 1]
    w64 = (bl[..., 2:].view(np.int8).astype(np.float64) * scale).reshape(n, k)
    dense = x.astype(np.float64) @ w64.T                                # [tokens, n]
    del w64
    err = np.linalg.norm(got.astype(np.float64) - dense, axis=1) / np.maximum(np.linalg.norm(dense, axis=1), 1e-30)
    assert err.max() < 1e-5, (int(err.argmax()), float(err.max()))
    for t in sorted({0, tokens // 2, tokens - 1}):
        ref = orc.q8_matmul(x[t], blocks.reshape(-1), n)
        assert rel_l2(got[t], ref) < 1e-5, t
