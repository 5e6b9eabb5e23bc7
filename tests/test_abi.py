"""The C-ABI library loads without a GPU, exports every function include/tir.h
declares, and its host-side pieces behave (no device work here)."""
import os
import re

import numpy as np
import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "tir.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tir_\w+)\s*\(", src)))


def test_library_exports_every_declared_function(tirlib):
    import ctypes
    names = declared_functions()
    assert len(names) >= 40
    raw = ctypes.CDLL(tirlib.LIB_PATH)
    missing = [n for n in names if not hasattr(raw, n)]
    assert not missing, missing


def test_binding_covers_the_header(tirlib):
    assert set(declared_functions()) == set(tirlib.SIGNATURES)


def test_version(tirlib):
    assert "sm100a" in tirlib.version()


@pytest.mark.parametrize("pos,dim,base", [(0, 64, 10000.0), (1, 4, 10000.0), (17, 64, 10000.0),
                                          (2047, 64, 10000.0), (513, 128, 500000.0)])
def test_rope_angles_host_is_bit_exact(tirlib, orc, pos, dim, base):
    np.testing.assert_array_equal(tirlib.rope_angles(base, pos, dim), orc.rope_angles(base, pos, dim))


def test_shape_errors_need_no_device(tirlib):
    with pytest.raises(tirlib.TirError) as e:
        tirlib.q8_matmul(0, 0, 0, 0, 4, 33)
    assert e.value.name == "UNSUPPORTED_SHAPE"
    with pytest.raises(tirlib.TirError) as e:
        tirlib.q8_repack(0, 4, 33, 0, 0)
    assert e.value.name == "BAD_QUANT_BLOCK"
    with pytest.raises(tirlib.TirError) as e:
        tirlib.embed(0, 10, 10, 64, 0)
    assert e.value.name == "BAD_TOKEN"
    with pytest.raises(tirlib.TirError) as e:
        tirlib.attention(0, 0, 0, 0, 8, 2, 32, 4, 16)
    assert e.value.name == "UNSUPPORTED_SHAPE"
    # the tensor-core matmul's activation planes cover rows of at most 6144
    with pytest.raises(tirlib.TirError) as e:
        tirlib.q8_matmul_batch(0, 4, (0, 0), 0, 128, 6144 + 64)
    assert e.value.name == "UNSUPPORTED_SHAPE"


def test_scale_stride(tirlib):
    assert tirlib.q8_scale_stride(2048) == 64
    assert tirlib.q8_scale_stride(5632) == 176
    assert tirlib.q8_scale_stride(1408) == 48  # 44 blocks padded to 16-byte rows
