"""Shared fixtures.  ``-m "not gpu"`` tests run anywhere (oracle, reader, ABI
surface); ``-m gpu`` tests need a B200 and call the CUDA path through the C ABI
(libtir.so), checking it against the CPU oracle."""
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tensor-inference-runtime_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU; calls the CUDA path via libtir.so")


@pytest.fixture(scope="session")
def kat():
    with open(os.path.join(GOLDEN, "reference_kat.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="session")
def orc():
    """The oracle in its fast mode (eight rows per pass, attention heads in
    parallel): the same bits as the reference's loop order, which
    tests/test_oracle_kat.py checks."""
    from oracle import load_oracle
    o = load_oracle()
    o.set_fast(True)
    return o


@pytest.fixture(scope="session")
def tirlib():
    import tir
    from tir import build
    if not os.path.exists(tir.LIB_PATH):
        build.build()
    tir.lib()
    return tir


@pytest.fixture(scope="session")
def cuda(tirlib):
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device (run them on the B200 box)"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) >= (10, 0), f"sm_100a kernels need compute capability 10.x, got {major}.{minor}"
    return torch


def _model(preset, seed=0):
    from tir import synth
    return synth.synthetic_model(preset, seed)


@pytest.fixture(scope="session")
def tiny_path():
    return _model("tiny")


@pytest.fixture(scope="session")
def small_path():
    return _model("small")


@pytest.fixture(scope="session")
def tinyllama_path():
    return _model("tinyllama")
