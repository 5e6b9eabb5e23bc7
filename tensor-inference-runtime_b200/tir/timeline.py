"""Summarises a decode phase timeline (State.trace()) per phase kind.

The trace holds, per phase and CTA, globaltimer stamps (start, inputs ready,
input staged, released), the ns thread 0 spent waiting for streamed weight
tiles, its tiles, and the ns it spent waiting for the previous phase.  For each
phase kind (qkv, attn, o, gu, down, lm) this reports, averaged over layers:

* barrier->ready: last release of the previous phase -> last CTA ready;
* staging: last CTA ready -> last CTA done staging its input;
* work: last staging done -> last release of the phase;
* data wait / dependency wait of thread 0, and its tile count.
"""
import numpy as np


def phase_names(n_phases):
    names = []
    for l in range((n_phases - 1) // 5):
        names += [f"L{l}.qkv", f"L{l}.attn", f"L{l}.o", f"L{l}.gu", f"L{l}.down"]
    return names + ["lm"]


def summarize(trace):
    tr = np.asarray(trace).astype(np.int64)
    P = tr.shape[0]
    names = phase_names(P)
    start = tr[:, :, 0][tr[:, :, 0] > 0].min()
    kinds = {}
    for p in range(P):
        r, st, e = tr[p, :, 1], tr[p, :, 2], tr[p, :, 3]
        prev_end = tr[p - 1, :, 3].max() if p else tr[p, :, 0].min()
        stv = st[st > 0]
        staged = stv.max() if stv.size else r.max()
        kinds.setdefault(names[p].split(".")[-1], []).append(
            ((r.max() - prev_end) / 1e3, (staged - r.max()) / 1e3, (e.max() - staged) / 1e3,
             tr[p, :, 4].mean() / 1e3, tr[p, :, 5].max(), tr[p, :, 6].mean() / 1e3))
    out = {"step_us": (tr[:, :, 3].max() - start) / 1e3, "kinds": {}}
    for k, v in kinds.items():
        v = np.array(v, np.float64)
        out["kinds"][k] = {"n": len(v), "barrier_to_ready_us": v[:, 0].mean(), "staging_us": v[:, 1].mean(),
                           "work_us": v[:, 2].mean(), "data_wait_us": v[:, 3].mean(),
                           "tiles_max": v[:, 4].mean(), "dep_wait_us": v[:, 5].mean()}
    return out


def to_markdown(summary):
    lines = [f"step: {summary['step_us']:.1f} us", "",
             "| phase | n | barrier->ready us | staging us | work us | data wait us | tiles (max CTA) | dep wait us |",
             "|---|---|---|---|---|---|---|---|"]
    for k, v in summary["kinds"].items():
        lines.append(f"| {k} | {v['n']} | {v['barrier_to_ready_us']:.2f} | {v['staging_us']:.2f} | {v['work_us']:.2f} | "
                     f"{v['data_wait_us']:.2f} | {v['tiles_max']:.1f} | {v['dep_wait_us']:.2f} |")
    return "\n".join(lines)
