"""Failure paths, driven in the forms that fault no GPU:

* a bounded device-side wait made to run out: a test hook makes one wait of
  the persistent decode kernel (or of a streaming matvec op) wait for a
  release that never comes, with a 1 ms limit; the launch must end with
  TIR_ERR_TIMEOUT, and the state (or the next op) must work normally after;
* allocation failure injected on the host: the n-th allocation of model load,
  state creation or batch creation fails, and each must return TIR_ERR_OOM
  (the reference's ModelLoadError covers the load step, src/error.rs:49-59),
  leak nothing and succeed on a clean retry.
"""
import ctypes as C

import numpy as np
import pytest

from tir import synth

pytestmark = pytest.mark.gpu

HOLD_US = 1000


def _n_phases(tirlib, st):
    n, g = C.c_int32(), C.c_int32()
    tirlib.check(tirlib.lib().tir_state_trace_dims(st.handle, C.byref(n), C.byref(g)))
    return n.value


def test_decode_wait_runs_out_then_state_recovers(cuda, tirlib, tiny_path):
    m = tirlib.Model(tiny_path)
    ref = m.state(max_ctx=16)
    ids = [5, 9, 11]
    want = [ref.forward(t, p) for p, t in enumerate(ids)]
    st = m.state(max_ctx=16)
    n_ph = _n_phases(tirlib, st)
    for phase in (1, 3, n_ph - 1):  # attention, output projection, lm_head waits
        st.forward(ids[0], 0)
        st.hold_phase(phase, HOLD_US)
        with pytest.raises(tirlib.TirError) as e:
            st.forward(ids[1], 1)
        assert e.value.name == "TIMEOUT" and f"phase {phase}," in str(e.value)
        assert len(st) == 0  # the cache was reset
        # the next launch decodes normally, bit for bit
        for p, t in enumerate(ids):
            np.testing.assert_array_equal(st.forward(t, p), want[p])
        st.reset()
    # a multi-step launch (generate_capped): phase 0 waits for the previous
    # step from the second step on, so the hold ends the launch in step 1
    st.hold_phase(0, HOLD_US)
    with pytest.raises(tirlib.TirError) as e:
        st.generate_capped(np.array(ids, np.int32), 4)
    assert e.value.name == "TIMEOUT" and "phase 0, step 1" in str(e.value)
    np.testing.assert_array_equal(st.generate_capped(np.array(ids, np.int32), 4),
                                  ref.generate_capped(np.array(ids, np.int32), 4))
    with pytest.raises(tirlib.TirError) as e:
        st.hold_phase(n_ph, HOLD_US)
    assert e.value.name == "INVALID_ARG"
    st.close()
    ref.close()
    m.close()


def _split(torch, tirlib, blocks, rows, k):
    b = torch.from_numpy(np.ascontiguousarray(blocks, np.uint8).reshape(-1).copy()).cuda()
    q = torch.empty(rows * k, dtype=torch.uint8, device="cuda")
    s = torch.empty(rows * tirlib.q8_scale_stride(k), dtype=torch.int16, device="cuda")
    tirlib.q8_repack(b, rows, k, q, s)
    return q, s


def test_op_wait_runs_out_is_reported_and_cleared(cuda, tirlib, orc):
    """An op whose wait gave up is reported by tir_ops_check (once), and it
    does not make later ops skip their work."""
    torch = cuda
    k, n = 2048, 2560
    x, blocks = synth.gemv_case(k, n, seed=21)
    want = orc.q8_matmul(x, blocks.reshape(-1), n)
    q, s = _split(torch, tirlib, blocks, n, k)
    dx = torch.from_numpy(x).cuda()
    tirlib.ops_check()  # nothing pending
    for _ in range(2):
        out = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
        tirlib.hold_next_op(HOLD_US)
        tirlib.q8_matmul(dx, q, s, out, n, k)
        with pytest.raises(tirlib.TirError) as e:
            tirlib.ops_check()
        assert e.value.name == "TIMEOUT"
        tirlib.ops_check()  # collected: clear now
        # the held launch finished its first pass before the wait
        got = out.cpu().numpy()
        assert np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want) < 1e-5
        # the next op runs in full and reports nothing
        out2 = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
        tirlib.q8_matmul(dx, q, s, out2, n, k)
        tirlib.ops_check()
        np.testing.assert_array_equal(out2.cpu().numpy(), got)


def _free_bytes(torch):
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0]


def _fail_each_allocation(tirlib, make):
    """make() with the n-th allocation failing, n = 0, 1, ... until it
    succeeds; every failure must be TIR_ERR_OOM.  Returns (object, failures)."""
    n = 0
    while True:
        tirlib.fail_alloc_after(n)
        try:
            obj = make()
        except tirlib.TirError as e:
            assert e.name == "OOM", (n, e)
            n += 1
            assert n < 200
            continue
        finally:
            tirlib.fail_alloc_after(-1)
        return obj, n


def test_allocation_failures_are_oom_without_leaks(cuda, tirlib, small_path):
    torch = cuda
    warm = tirlib.Model(small_path)  # context, per-device buffers, kernel attributes
    ws = warm.state(max_ctx=8)
    want = ws.forward(7, 0)
    ws.close()
    warm.close()
    free0 = _free_bytes(torch)
    slack = 16 << 20

    m, n_model = _fail_each_allocation(tirlib, lambda: tirlib.Model(small_path))
    assert n_model >= 2  # weights, upload staging
    st, n_state = _fail_each_allocation(tirlib, lambda: m.state(max_ctx=8192))
    assert n_state >= 10
    b, n_batch = _fail_each_allocation(tirlib, lambda: tirlib.Batch(m, 4, max_ctx=2048, max_tokens_per_seq=8))
    assert n_batch >= 10
    # the clean retries work
    np.testing.assert_array_equal(st.forward(7, 0), want)
    nxt = b.step(np.array([[1], [2], [3], [4]], np.int32))
    assert nxt.shape == (4,)
    b.close()
    st.close()
    m.close()
    # nothing the failed attempts allocated is still held
    assert _free_bytes(torch) >= free0 - slack
    before = tirlib.alloc_count()
    tirlib.fail_alloc_after(0)
    with pytest.raises(tirlib.TirError) as e:
        tirlib.Model(small_path)
    assert e.value.name == "OOM"
    assert tirlib.alloc_count() == before + 1  # stopped at the first failure
    tirlib.fail_alloc_after(-1)
