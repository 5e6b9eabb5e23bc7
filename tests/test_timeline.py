"""tir.timeline on a hand-made trace (no GPU): the per-phase-kind figures the
decode kernel's phase timeline reports, from the stamps it records."""
import numpy as np

from tir import timeline


def _trace(layers=2, grid=3):
    """Phases of `layers` layers (5 kinds each) + lm, `grid` CTAs, 8 fields:
    every phase starts 10 ns after the previous release, inputs are ready 100 ns
    later (the last CTA), staged 50 ns later, released 400 ns later."""
    P = 5 * layers + 1
    tr = np.zeros((P, grid, 8), np.uint64)
    t = 1_000
    for p in range(P):
        for c in range(grid):
            tr[p, c, 0] = t + 10
            tr[p, c, 1] = t + 100 + c  # the last CTA is ready at t + 100 + grid - 1
            tr[p, c, 2] = t + 150 + grid
            tr[p, c, 3] = t + 550 + grid
            tr[p, c, 4] = 20 * (c + 1)  # ns waiting for ring data
            tr[p, c, 5] = c + 1         # tiles
            tr[p, c, 6] = 30            # ns waiting for the previous phase
        t = int(tr[p, :, 3].max())
    return tr


def test_phase_names_cover_every_phase():
    names = timeline.phase_names(11)
    assert names[:5] == ["L0.qkv", "L0.attn", "L0.o", "L0.gu", "L0.down"] and names[-1] == "lm"
    assert len(names) == 11


def test_summary_figures():
    tr = _trace()
    s = timeline.summarize(tr)
    k = s["kinds"]
    assert set(k) == {"qkv", "attn", "o", "gu", "down", "lm"}
    assert k["qkv"]["n"] == 2 and k["lm"]["n"] == 1
    # the previous release -> the last CTA ready: 100 + grid - 1 ns
    assert np.isclose(k["gu"]["barrier_to_ready_us"], (100 + 2) / 1e3)
    assert np.isclose(k["gu"]["staging_us"], (150 + 3 - 102) / 1e3)
    assert np.isclose(k["gu"]["work_us"], 400 / 1e3)
    assert np.isclose(k["down"]["data_wait_us"], 40 / 1e3)  # mean of 20, 40, 60 ns
    assert k["down"]["tiles_max"] == 3
    assert np.isclose(k["o"]["dep_wait_us"], 0.03)
    assert np.isclose(s["step_us"], (tr[:, :, 3].max() - tr[0, :, 0].min()) / 1e3)
    md = timeline.to_markdown(s)
    assert md.startswith("step: ") and "| gu | 2 |" in md
