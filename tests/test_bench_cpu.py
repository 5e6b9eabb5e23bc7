"""bench.py's host-side arithmetic (no GPU): the algorithmic bytes behind the
batch-1 roofline, pinned to the TinyLlama-shape figures (1,099,442,304 B per
forward: every Q8_0 quant and f16 scale, the norm weights and one embedding
row), and the workload arguments."""
import bench

TINYLLAMA = {"embed_dim": 2048, "kv_dim": 256, "layers": 22, "ffn_dim": 5632, "vocab": 32000}


def q8_bytes(n, k):
    return n * k + n * (k // 32) * 2  # int8 quants + one f16 scale per 32


def tinyllama_weight_bytes():
    H, KVD, F, V, L = (TINYLLAMA[k] for k in ("embed_dim", "kv_dim", "ffn_dim", "vocab", "layers"))
    layer = q8_bytes(H + 2 * KVD, H) + q8_bytes(H, H) + q8_bytes(2 * F, H) + q8_bytes(H, F) + 2 * H * 4
    return L * layer + q8_bytes(V, H) + H * 4


def test_weight_bytes_per_forward():
    assert tinyllama_weight_bytes() + 2048 + 2048 // 32 * 2 == 1_099_442_304


def test_algorithmic_bytes_of_the_default_workload():
    # 16 prompt ids + 128 greedy steps: 144 forwards, each the weights plus the
    # KV cache read at positions 0..pos and written at pos (45,056 B a position)
    alg = bench.algorithmic_bytes(TINYLLAMA, tinyllama_weight_bytes(), 144)
    kv = 2 * 22 * 256 * 4
    assert kv == 45_056
    assert alg == 144 * 1_099_442_304 + kv * sum(pos + 2 for pos in range(144)) == 158_796_564_480


def test_workload_arguments():
    a = bench.parse_args([])
    assert (a.prompt, a.decode, a.gpus, a.workload) == (16, 128, 1, "decode") and a.warmup >= 3
    assert bench.workload_name(a) == bench.WORKLOAD
    b = bench.parse_args(["--workload", "long"])
    assert (b.prompt, b.decode) == (1792, 256)
    assert "1792-token seeded prompt + 256 steps (2048 forwards per step)" in bench.workload_name(b)


def test_committed_traffic_follows_the_build(tmp_path, monkeypatch):
    """A committed ncu traffic figure is used only on the decode-kernel build
    (source hash) and workload it was captured on."""
    import json
    import os
    sha = bench.decode_source_sha()
    assert len(sha) == 16 and sha == bench.decode_source_sha()
    prof = tmp_path / "profiles"
    prof.mkdir()
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    assert bench.committed_traffic(16, 128)[0] is None
    rec = {"prompt": 16, "decode": 128, "bytes_per_launch": 123, "source_sha": sha}
    (prof / "decode_traffic.json").write_text(json.dumps(rec))
    assert bench.committed_traffic(16, 128)[0] == 123
    assert bench.committed_traffic(1792, 256)[0] is None
    rec["source_sha"] = "0" * 16
    (prof / "decode_traffic.json").write_text(json.dumps(rec))
    assert bench.committed_traffic(16, 128)[0] is None
    assert os.path.exists(os.path.join(bench.PKG, "csrc", "decode.cu"))
