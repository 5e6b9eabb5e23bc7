"""tir_swiglu_static (intermediates in a fixed per-device array, no device
allocation) against tir_swiglu (per-call scratch) on the same inputs, two calls
in a row, plus its size limit.  The file name sorts last so the test also runs
after every other GPU test in a full session."""
import numpy as np
import pytest

from tir import synth

pytestmark = pytest.mark.gpu


def _dev(torch, a):
    return torch.from_numpy(np.array(a, copy=True)).cuda()


def _split(torch, tirlib, blocks, rows, k):
    b = _dev(torch, np.ascontiguousarray(blocks, np.uint8).reshape(-1))
    q = torch.empty(rows * k, dtype=torch.uint8, device="cuda")
    s = torch.empty(rows * tirlib.q8_scale_stride(k), dtype=torch.int16, device="cuda")
    tirlib.q8_repack(b, rows, k, q, s)
    return q, s


def _ffn(torch, tirlib, k, f, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(k).astype(np.float32)
    _, wg = synth.gemv_case(k, f, seed=seed + 1)
    _, wu = synth.gemv_case(k, f, seed=seed + 2)
    _, wd = synth.gemv_case(f, k, seed=seed + 3)
    return (x, wg, wu, wd), (_dev(torch, x), _split(torch, tirlib, wg, f, k), _split(torch, tirlib, wu, f, k),
                             _split(torch, tirlib, wd, k, f))


@pytest.mark.parametrize("k,f", [(2048, 5632), (256, 6144)])
def test_swiglu_static_matches_swiglu_twice(cuda, tirlib, orc, k, f):
    torch = cuda
    calls = []
    for seed in (31, 57):  # two calls in a row, different inputs, same static scratch
        (x, wg, wu, wd), (dx, g, u, d) = _ffn(torch, tirlib, k, f, seed)
        want = torch.empty(k, dtype=torch.float32, device="cuda")
        got = torch.full((k,), float("nan"), dtype=torch.float32, device="cuda")
        n0 = tirlib.alloc_count()
        tirlib.swiglu(dx, g, u, d, want, k, f)
        n1 = tirlib.alloc_count()
        tirlib.swiglu_static(dx, g, u, d, got, k, f)
        # the library's allocation counter sees tir_swiglu's per-call scratch
        # and nothing from the static entry
        assert n1 == n0 + 1 and tirlib.alloc_count() == n1
        tirlib.ops_check()  # no device-side wait gave up
        torch.cuda.synchronize()
        calls.append((got.cpu().numpy(), want.cpu().numpy(), orc.swiglu(x, wg.reshape(-1), wu.reshape(-1),
                                                                          wd.reshape(-1), f)))
    for got, want, ref in calls:
        np.testing.assert_array_equal(got, want)  # same kernels, same inputs: identical bits
        assert np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref) < 1e-5
    assert not np.array_equal(calls[0][0], calls[1][0])


def test_swiglu_static_rejects_sizes_above_its_scratch(cuda, tirlib):
    torch = cuda
    k, f = 64, 6144 + 32
    x = torch.zeros(k, dtype=torch.float32, device="cuda")
    q = torch.zeros(f * k, dtype=torch.uint8, device="cuda")
    s = torch.zeros(f * tirlib.q8_scale_stride(max(k, f)), dtype=torch.int16, device="cuda")
    out = torch.zeros(k, dtype=torch.float32, device="cuda")
    with pytest.raises(tirlib.TirError) as e:
        tirlib.swiglu_static(x, (q, s), (q, s), (q, s), out, k, f)
    assert e.value.status == 24 and "static scratch" in str(e.value)
