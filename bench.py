#!/usr/bin/env python
"""Batch-1 Q8_0 Llama-2 decode benchmark (TinyLlama-1.1B shape, synthetic GGUF).

One step = one generate_capped over the workload: a 16-token seeded prompt fed
token by token, then 128 greedy decode steps -- 144 forward passes, each
streaming the 1.10 GB of Q8_0 weights from HBM (every forward also computes the
logits, as the reference does).  The whole loop runs on the device in one
persistent-kernel launch.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

The default run also measures the other workloads of the same model, each in
its own timed region, as sub-objects of the one JSON line: "long" (1792 prompt
ids + 256 greedy steps, context 2048), "batched" (64 sequences per GPU x (128
prompt ids + 128 greedy steps) on the tensor-core path), "prefill" (16 x 512
prompt ids per GPU in one batched forward) and, on rank 0, "gemv" (the
isolated Q8_0 GEMV sweep over the five projection shapes).  --sub off skips
them; --workload NAME runs one of them alone as the headline.

N > 1 runs under torchrun, one process per GPU; each GPU holds a full weight
replica and decodes its own sequences (replicas, no collective on the data
path; torch.distributed only brackets the timed regions).  Rank 0 prints one
JSON line; every value is the aggregate over ranks (tokens of all ranks / the
slowest rank's device time).

--impl reference times the oracle -- the C restatement of the reference's
Rayon CPU path -- on the host cores of rank 0 only, on a bounded sample of
the same workload (not scaled with N).
"""
import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "tensor-inference-runtime_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

WORKLOAD = ("TinyLlama-1.1B-shape Llama-2 decoder (22 layers, hidden 2048, 32/4 heads, "
            "FFN 5632, vocab 32000) as a synthetic Q8_0 GGUF; batch-1 greedy decode of a "
            "16-token seeded prompt + 128 steps (144 forwards per step)")
METRIC = "decode tok/s (batch 1)"


def workload_name_for(n_prompt, n_decode):
    if n_prompt == 16 and n_decode == 128:
        return WORKLOAD
    return WORKLOAD.replace("16-token seeded prompt + 128 steps (144 forwards per step)",
                            f"{n_prompt}-token seeded prompt + {n_decode} steps "
                            f"({n_prompt + n_decode} forwards per step)")


def workload_name(args):
    return workload_name_for(args.prompt, args.decode)


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prompt", type=int, default=16)
    ap.add_argument("--decode", type=int, default=128)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-baseline", choices=["auto", "off"], default="auto")
    ap.add_argument("--workload", choices=["decode", "long", "gemv", "batched", "prefill"], default="decode",
                    help="decode: the batch-1 decode loop, 16 prompt ids + 128 steps (default); long: the same "
                         "loop with a 1792-id prompt + 256 steps (context 2048); gemv: the isolated Q8_0 GEMV "
                         "sweep over the TinyLlama projection shapes; batched: 64 sequences per GPU, 128 prompt "
                         "ids + 128 greedy steps each, on the tensor-core path; prefill: 16 sequences x 512 prompt "
                         "ids per GPU in one batched forward")
    ap.add_argument("--sub", choices=["on", "off"], default="on",
                    help="with the default decode workload: also measure the long, batched, prefill and GEMV "
                         "workloads as sub-objects of the line")
    ap.add_argument("--timeline", metavar="FILE.md", default=None,
                    help="after the timed region, trace one forward step (--timeline-step) of one more "
                         "generate and write the per-phase timeline summary to FILE.md")
    ap.add_argument("--timeline-step", type=int, default=100,
                    help="the traced forward step (0-based; clamped to the generate's last step)")
    args = ap.parse_args(argv)
    if args.workload == "long":
        args.prompt, args.decode = 1792, 256
    return args


# ---------------------------------------------------------------------------
# distributed plumbing (barrier + max over ranks); no collective on the data path
# ---------------------------------------------------------------------------
def decode_seed(seed, rank):
    """Prompt seed of rank `rank`'s batch-1 sequence (each rank its own)."""
    return seed + rank


def batched_seed(seed, rank):
    """Seed of rank `rank`'s batch of sequences (each rank its own shard)."""
    return seed + 7919 * rank


class Dist:
    def __init__(self, backend="nccl"):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch
            import torch.distributed as dist
            kw = {"device_id": torch.device("cuda", self.local)} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=180), **kw)
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v):
        if not self.pg:
            return v
        import torch
        dev = "cuda" if self.pg.get_backend() == "nccl" else "cpu"
        t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        # nvidia-smi's start-up can hold the driver for seconds: the timed
        # region opens only once it delivers samples (at most 10 s)
        t0 = time.perf_counter()
        while self.proc and not self.rows and self.proc.poll() is None and time.perf_counter() - t0 < 10.0:
            time.sleep(0.01)
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and (not self.uuid or self.uuid in parts[0]):
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------------------
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def algorithmic_bytes(info, weight_bytes, n_forwards):
    """Bytes one generate must move: every forward streams all weights (quants,
    scales, norms) plus one embedding row, reads the KV cache of positions
    0..pos and writes position pos (4-byte floats, K and V, every layer)."""
    H = info["embed_dim"]
    emb_row = H + H // 32 * 2
    kv_pos = 2 * info["layers"] * info["kv_dim"] * 4
    total = 0
    for pos in range(n_forwards):
        total += weight_bytes + emb_row + kv_pos * (pos + 1) + kv_pos
    return total


def host_threads():
    """Host cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, dist):
    """The oracle (C restatement of the reference's Rayon path) on host cores."""
    import numpy as np
    from oracle import load_oracle
    from oracle.gguf_ref import GGUF
    from tir import synth

    path = synth.synthetic_model("tinyllama", args.seed)
    orc = load_oracle()
    orc.set_threads(host_threads())  # torchrun sets OMP_NUM_THREADS=1; use every host core
    om = orc.model(GGUF(path))
    prompt = synth.prompt_ids(args.prompt, 32000, seed=args.seed)
    # bounded sample per step: 4 forwards (2 prompt ids + 2 greedy) at the
    # workload's start; per-token cost is flat at this context length
    sample_prompt, sample_cap = prompt[:2], 2
    for _ in range(args.warmup):
        om.generate_capped(sample_prompt, sample_cap)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        om.generate_capped(sample_prompt, sample_cap)
    dt = (time.perf_counter() - t0) / args.steps
    value = (len(sample_prompt) + sample_cap) / dt
    sample = (f"{len(sample_prompt)} prompt ids + {sample_cap} greedy steps of the workload per step (positions "
              f"0-{len(sample_prompt) + sample_cap - 1}: at these context lengths the reference's per-token cost is "
              f"flat, so the rate stands for the whole workload's); one process on rank 0's host, not scaled with N")
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Q8_0 weights and token ids)",
            "config": {"workload": workload_name(args), "batch": 1, "prompt_tokens": args.prompt,
                       "decode_tokens": args.decode, "parallelism": "host cores of rank 0 (one process at any N)"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": orc.get_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline(args):
    """Oracle timed on the host cores on a bounded sample (rank 0, N=1)."""
    from oracle import load_oracle
    from oracle.gguf_ref import GGUF
    from tir import synth
    path = synth.synthetic_model("tinyllama", args.seed)
    orc = load_oracle()
    orc.set_threads(host_threads())
    om = orc.model(GGUF(path))
    prompt = synth.prompt_ids(args.prompt, 32000, seed=args.seed)
    om.generate_capped(prompt[:1], 0)  # page the weights in
    n_prompt, cap = 8, 8
    t0 = time.perf_counter()
    om.generate_capped(prompt[:n_prompt], cap)
    dt = time.perf_counter() - t0
    return {"value": (n_prompt + cap) / dt, "unit": "tok/s", "cores": orc.get_threads(), "kind": "port",
            "sample": f"first {n_prompt} prompt ids + {cap} greedy steps of the workload (16 forwards)"}


def cpu_baseline_batched(args):
    """Oracle on the host cores for the batched workloads, on the samples the
    measurement plan names: the batched decode workload on 2 of its sequences
    (each 128 prompt ids + 128 greedy steps), the prefill workload on one of
    its 512-id sequences -- the reference runs sequences one after another and
    feeds prompts token by token, so tok/s = forwards / wall time."""
    from oracle import load_oracle
    from oracle.gguf_ref import GGUF
    from tir import synth
    import numpy as np
    orc = load_oracle()
    orc.set_threads(host_threads())
    om = orc.model(GGUF(synth.synthetic_model("tinyllama", args.seed)))
    rng = np.random.default_rng(args.seed)
    if args.workload == "batched":
        seqs, P, cap = 2, 128, args.decode
        sample = f"2 of the 64 sequences, each {P} prompt ids + {cap} greedy steps ({seqs * (P + cap)} forwards)"
    else:
        seqs, P, cap = 1, 512, 0
        sample = "one of the 16 sequences: 512 prompt ids fed token by token (512 forwards)"
    prompts = rng.integers(3, 32000, size=(seqs, P), dtype=np.int32)
    om.generate_capped(prompts[0, :1], 0)  # page the weights in
    t0 = time.perf_counter()
    for s_ in range(seqs):
        om.generate_capped(prompts[s_], cap)
    dt = time.perf_counter() - t0
    return {"value": seqs * (P + cap) / dt, "unit": "tok/s", "cores": orc.get_threads(), "kind": "port",
            "sample": sample}


def decode_source_sha():
    """First 16 hex digits of the sha256 of the decode kernel's sources: a
    committed ncu traffic figure applies only to the build it was taken on."""
    h = hashlib.sha256()
    for name in ("decode.cu", "runtime.h", "ptx.cuh"):
        with open(os.path.join(PKG, "csrc", name), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def committed_traffic(n_prompt, n_decode):
    """DRAM bytes of one decode launch from profiles/decode_traffic.json when it
    was taken on this workload and on these decode-kernel sources, else None."""
    tpath = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if not os.path.exists(tpath):
        return None, "no committed capture"
    with open(tpath) as f:
        t = json.load(f)
    if t.get("prompt") != n_prompt or t.get("decode") != n_decode:
        return None, "committed capture is of another workload"
    if t.get("source_sha") != decode_source_sha():
        return None, "committed capture is of another build of the decode kernel"
    return t.get("bytes_per_launch"), "ncu capture of this build (profiles/decode_traffic.json)"


def measure_decode(model, dist, n_prompt, n_decode, steps, warmup, seed, timeline=None, timeline_step=100):
    """generate_capped of n_prompt seeded ids + n_decode greedy steps, one
    launch per step: device time with the prompt resident in HBM (CUDA events
    on the state's stream, max over ranks), then end to end through the host
    API (host ids in and out).  Returns the JSON fields of the measurement."""
    import torch

    from tir import synth

    dev = dist.local
    info = model.info
    n_fwd = n_prompt + n_decode
    st = model.state(max_ctx=n_fwd)
    stream = torch.cuda.ExternalStream(st.stream(), device=torch.device("cuda", dev))
    # each rank decodes its own sequence (weak scaling)
    prompt = synth.prompt_ids(n_prompt, info["vocab"], seed=decode_seed(seed, dist.rank))
    d_prompt = torch.from_numpy(prompt.copy()).to(f"cuda:{dev}")
    d_out = torch.empty(n_decode, dtype=torch.int32, device=f"cuda:{dev}")

    def step():
        st.generate_capped_device(d_prompt, n_prompt, n_decode, d_out)

    for _ in range(warmup):
        step()
    st.sync()

    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", "")) or None
    # ---- device-timed region (inputs resident in HBM) -----------------------
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(uuid) as clocks:
        time.sleep(0.05)
        ev[0].record(stream)
        for i in range(steps):
            step()
            ev[i + 1].record(stream)
        torch.cuda.synchronize(dev)
    st.sync()
    ms_local = sum(ev[i].elapsed_time(ev[i + 1]) for i in range(steps)) / steps
    dist.barrier()
    ms = dist.max(ms_local)

    # ---- end to end through the host API (host ids in and out) -------------
    for _ in range(max(1, warmup // 2)):
        st.generate_capped(prompt, n_decode)
    dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(steps):
        ids = st.generate_capped(prompt, n_decode)
    torch.cuda.synchronize(dev)
    e2e_local = (time.perf_counter() - t0) / steps * 1e3
    dist.barrier()
    e2e_ms = dist.max(e2e_local)
    assert ids.shape == (n_decode,)

    total_tokens = n_fwd * dist.world
    peak, peak_kind = peaks()
    alg = algorithmic_bytes(info, model.weight_bytes(), n_fwd)
    achieved = alg / (ms_local / 1e3) / 1e9
    traffic, traffic_src = committed_traffic(n_prompt, n_decode)
    out = {
        "value": total_tokens / (ms / 1e3), "unit": "tok/s", "steps": steps, "warmup": warmup, "ms_per_step": ms,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_src,
                     "peak_kind": peak_kind, "kernel": "tir::decode_kernel (one launch per step)",
                     "algorithmic_bytes_per_launch": alg},
        "e2e": {"value": total_tokens / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": 4 * n_prompt,
                "d2h_bytes_per_step": 4 * n_decode + 12},
        "gpu_launches": steps,
        "clocks": clocks.summary(),
    }
    if timeline and dist.rank == 0:
        from tir import timeline as tl
        st.enable_trace(min(max(timeline_step, 0), n_fwd - 1))
        st.generate_capped(prompt, n_decode)
        st.enable_trace(-1)
        with open(timeline, "w") as f:
            f.write(tl.to_markdown(tl.summarize(st.trace())) + "\n")
    st.close()
    return out


def decode_config(n_prompt, n_decode, world):
    return {"workload": workload_name_for(n_prompt, n_decode), "batch": 1, "prompt_tokens": n_prompt,
            "decode_tokens": n_decode, "forwards_per_step": n_prompt + n_decode,
            "parallelism": f"replicas x{world} (no collective)",
            "l2": "inputs larger than L2: 1.10 GB of weights streamed per forward vs 126 MB L2"}


def run_ours(args, dist):
    import torch

    import tir
    from tir import synth

    dev = dist.local
    torch.cuda.set_device(dev)
    if dist.rank == 0:
        synth.synthetic_model("tinyllama", args.seed)
    dist.barrier()
    model = tir.Model(synth.synthetic_model("tinyllama", args.seed), device=dev)
    m = measure_decode(model, dist, args.prompt, args.decode, args.steps, args.warmup, args.seed, args.timeline,
                       args.timeline_step)
    line = {"metric": METRIC, "value": m["value"], "unit": "tok/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": m["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Q8_0 weights and token ids)",
            "config": decode_config(args.prompt, args.decode, dist.world)}
    for k in ("roofline", "e2e", "gpu_launches", "clocks"):
        line[k] = m[k]
    if dist.rank == 0 and dist.world == 1 and args.cpu_baseline == "auto":
        line["cpu_baseline"] = cpu_baseline(args)
    if args.sub == "on" and args.workload == "decode" and (args.prompt, args.decode) == (16, 128):
        # the other workloads of the same model, each in its own timed region
        sub_steps, sub_warm = max(1, min(args.steps, 3)), max(3, min(args.warmup, 3))
        long_m = measure_decode(model, dist, 1792, 256, sub_steps, sub_warm, args.seed)
        line["long"] = dict(metric="decode tok/s (batch 1, context 2048)", config=decode_config(1792, 256, dist.world),
                            **long_m)
        for kind in ("batched", "prefill"):
            line[kind] = measure_batched(model, dist, kind, 128, sub_steps, sub_warm, args.seed)
        if dist.rank == 0:
            line["gemv"] = measure_gemv(dev, sub_steps, sub_warm, args.seed)
            line["gemv"]["ranks"] = "rank 0 only (a per-GPU figure)"
    model.close()
    return line


GEMV_SHAPES = [(2048, 2048), (2048, 256), (2048, 5632), (5632, 2048), (2048, 32000)]  # (K, N)


def measure_gemv(dev, steps, warmup, seed):
    """Isolated Q8_0 GEMV sweep (batch 1) over the TinyLlama projection shapes:
    x f32 N(0, 1), weights int8 uniform in [-127, 127] with f16 scales
    |N(0, 0.02)| / 127, seeded, in the tile-major layout the decode kernel
    streams; each launch reads the next of several weight copies (>= 4x the
    126 MB L2 in total) so weights stream from HBM.  Value = weight bytes
    (N K / 32 x 34) over the summed device time of all shapes."""
    import torch

    import tir
    torch.cuda.set_device(dev)
    g = torch.Generator(device="cuda").manual_seed(seed)
    l2 = 126 * 2 ** 20
    per_shape = []
    tot_bytes, tot_ms = 0.0, 0.0
    stream = torch.cuda.current_stream()
    for k, n in GEMV_SHAPES:
        nb = k // 32
        wbytes = n * nb * 34
        tiled = tir.q8_tiled_bytes(n, k)
        copies = max(2, -(-4 * l2 // tiled))
        ws = []
        for _ in range(copies):
            q = torch.randint(-127, 128, (n, nb, 32), dtype=torch.int8, device="cuda", generator=g)
            sc = (torch.randn(n, nb, 1, device="cuda", generator=g).abs() * 0.02 / 127).half()
            blocks = torch.cat([sc.view(torch.uint8), q.view(torch.uint8)], dim=2).contiguous()
            w = torch.empty(tiled, dtype=torch.uint8, device="cuda")
            tir.q8_repack_tiled(blocks, n, k, w)
            ws.append(w)
            del q, sc, blocks
        x = torch.randn(k, device="cuda", generator=g)
        out = torch.empty(n, device="cuda")
        for i in range(max(warmup, 3) * copies):
            tir.q8_matmul_tiled(x, ws[i % copies], out, n, k)
        iters = max(steps, 1) * copies
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(iters):
            tir.q8_matmul_tiled(x, ws[i % copies], out, n, k)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        per_shape.append({"k": k, "n": n, "us": ms * 1e3, "weight_gbs": wbytes / (ms / 1e3) / 1e9, "copies": copies})
        tot_bytes += wbytes
        tot_ms += ms
        del ws
    peak, peak_kind = peaks()
    gbs = tot_bytes / (tot_ms / 1e3) / 1e9
    line = {"metric": "Q8_0 GEMV weight GB/s (batch 1, TinyLlama projection shapes)", "value": gbs, "unit": "GB/s",
            "n_gpus": 1, "steps": steps, "warmup": warmup, "ms_per_step": tot_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded int8 weights, f16 scales, f32 activations)",
            "config": {"workload": "Q8_0 GEMV sweep K->N: " + ", ".join(f"{k}->{n}" for k, n in GEMV_SHAPES),
                       "l2": "each launch reads the next of >= 4x L2 of weight copies"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "traffic": None, "peak_kind": peak_kind},
            "shapes": per_shape, "gpu_launches": sum(max(steps, 1) * s["copies"] for s in per_shape)}
    return line


def run_gemv(args):
    print(json.dumps(measure_gemv(0, args.steps, args.warmup, args.seed)), flush=True)


def measure_batched(model, dist, kind, decode_cap, steps, warmup, seed, cpu=None):
    """Batched sequences on the tensor-core path (one process per GPU, weak
    scaling).  batched: 64 sequences x (128 seeded prompt ids + decode_cap
    greedy steps), value = all token forwards / device time of one generate;
    prefill: 16 sequences x 512 seeded ids in one batched forward, value =
    prompt tokens / device time.  cpu: the arguments of the oracle's CPU
    baseline for this workload (rank 0, N = 1), or None."""
    import numpy as np
    import torch

    import tir

    dev = dist.local
    info = model.info
    V = info["vocab"]
    if kind == "batched":
        B, P, cap = 64, 128, decode_cap
    else:
        B, P, cap = 16, 512, 0
    rng = np.random.default_rng(batched_seed(seed, dist.rank))
    prompts = rng.integers(3, V, size=(B, P), dtype=np.int32)
    batch = tir.Batch(model, B, max_ctx=P + cap + 1, max_tokens_per_seq=P)
    stream = torch.cuda.ExternalStream(batch.stream(), device=torch.device("cuda", dev))

    def step():
        if kind == "batched":
            return batch.generate(prompts, cap)
        batch.reset()
        return batch.step(prompts)

    for _ in range(warmup):
        step()
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", "")) or None
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(uuid) as clocks:
        t0 = time.perf_counter()  # after the sampler's start-up, which is not the workload's
        ev[0].record(stream)
        for i in range(steps):
            step()
            ev[i + 1].record(stream)
        torch.cuda.synchronize(dev)
        wall_ms = (time.perf_counter() - t0) / steps * 1e3
    ms_local = sum(ev[i].elapsed_time(ev[i + 1]) for i in range(steps)) / steps
    dist.barrier()
    ms = dist.max(ms_local)
    e2e_ms = dist.max(wall_ms)
    forwards = P + cap
    tokens = B * forwards * dist.world
    # kernels of one step: a multi-token forward is the embedding, 10 per layer
    # (norm planes, q|k|v matmul, RoPE + KV append, attention, planes, o
    # matmul, norm planes, gate|up matmul, SiLU planes, down matmul) and 4 at
    # the end (last rows, final norm planes, lm_head matmul, argmax); a decode
    # forward has no separate RoPE launch, plus the id feedback kernel
    L_ = info["layers"]
    launches_per_step = (1 + 10 * L_ + 4) + cap * (1 + 9 * L_ + 4 + 1)
    wb = model.weight_bytes()
    if kind == "batched":
        name = (f"TinyLlama-1.1B-shape Q8_0 model, {B} sequences per GPU, each {P} seeded prompt ids (one batched "
                f"prefill) + {cap} greedy steps in lockstep ({B * forwards} token forwards per step)")
        kv_pos = 2 * info["layers"] * info["kv_dim"] * 4
        alg = (1 + cap) * wb + B * sum(kv_pos * (pos + 1) + kv_pos for pos in range(P, P + cap)) + \
            B * P * kv_pos * 2
        peak, kind = peaks()
        roof = {"bound": "hbm", "achieved": alg / (ms_local / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                "frac": alg / (ms_local / 1e3) / 1e9 / peak, "traffic": None, "peak_kind": kind,
                "kernel": "tensor-core Q8_0 matmul + batched attention (one launch sequence per step)",
                "algorithmic_bytes_per_step": alg}
        metric = "batched decode tok/s (64 sequences per GPU, aggregate)"
    else:
        name = (f"TinyLlama-1.1B-shape Q8_0 model, {B} sequences x {P} seeded prompt ids per GPU in one batched "
                f"forward (M = {B * P} rows per matmul)")
        H, KVD, F, L = info["embed_dim"], info["kv_dim"], info["ffn_dim"], info["layers"]
        per_token = L * (H * (H + 2 * KVD) + H * H + 2 * F * H + F * H)  # 968,884,224 for TinyLlama
        flops = 2.0 * per_token * B * P + 2.0 * V * H * B
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                mp = json.load(f)
            peak, kind = float(mp.get("bf16_tflops_sustained", mp["bf16_tflops"])), "measured"
        except (OSError, KeyError, ValueError):
            peak, kind = 1590.0, "fallback"
        ach = flops / (ms_local / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                "traffic": None, "peak_kind": kind,
                "kernel": "tir gemm_q8_kernel (tcgen05 kind::f16, 3 passes; algorithmic FLOPs counted once)",
                "algorithmic_flops_per_step": flops}
        metric = "prefill tok/s (16 x 512 tokens per GPU, aggregate)"
    line = {"metric": metric, "value": tokens / (ms / 1e3), "unit": "tok/s", "n_gpus": dist.world,
            "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (3-pass f16 tensor cores, f32 accumulation)",
            "data": "synthetic (seeded Q8_0 weights and token ids)",
            "config": {"workload": name, "sequences_per_gpu": B, "prompt_tokens": P, "decode_tokens": cap,
                       "parallelism": f"replicas x{dist.world} (no collective)",
                       "l2": "inputs larger than L2: 1.10 GB of weights per forward step vs 126 MB L2"},
            "roofline": roof,
            "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": B * P * 4,
                    "d2h_bytes_per_step": B * cap * 4 + 4},
            "gpu_launches": steps * launches_per_step, "clocks": clocks.summary()}
    batch.close()
    if cpu is not None and dist.world == 1:
        line["cpu_baseline"] = cpu_baseline_batched(cpu)
    return line


def run_batched(args, dist):
    import torch

    import tir
    from tir import synth

    dev = dist.local
    torch.cuda.set_device(dev)
    if dist.rank == 0:
        synth.synthetic_model("tinyllama", args.seed)
    dist.barrier()
    model = tir.Model(synth.synthetic_model("tinyllama", args.seed), device=dev)
    line = measure_batched(model, dist, args.workload, args.decode, args.steps, args.warmup, args.seed,
                           cpu=args if args.cpu_baseline == "auto" else None)
    model.close()
    return line


def main(argv=None):
    args = parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank = int(os.environ.get("RANK", 0))
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, None)
        return 0
    if args.workload == "gemv":
        if rank == 0:
            run_gemv(args)
        return 0
    dist = Dist("nccl")
    try:
        line = run_batched(args, dist) if args.workload in ("batched", "prefill") else run_ours(args, dist)
        if dist.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
