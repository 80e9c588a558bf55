"""Shared fixtures.  GPU tests are marked `gpu` and call the CUDA path through the C ABI."""
import importlib
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def g4():
    return importlib.import_module("gemma4-js_b200")


@pytest.fixture(scope="session")
def rt():
    return importlib.import_module("gemma4-js_b200.runtime")


@pytest.fixture(scope="session")
def oracle():
    return importlib.import_module("oracle")


@pytest.fixture(scope="session")
def npo():
    return importlib.import_module("oracle.numpy_oracle")


@pytest.fixture(scope="session")
def ctx(rt):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = rt.Context(0)
    yield c
    c.sync()


@pytest.fixture(scope="session")
def ops(rt, ctx):
    return rt.GPUOps(ctx)


def golden(name):
    d = np.load(GOLDEN / name)
    return {k: d[k] for k in d.files}


def bf16_round(x):
    """f32 -> nearest-even bf16 value as f32 (the value a bf16 tensor holds)."""
    o = importlib.import_module("oracle")
    return o.bf16_bits_to_f32(o.f32_to_bf16_bits(np.asarray(x, np.float32)))


def max_rel(y, ref):
    """max|y - ref| / max|ref| (the tolerance metric of the hot path's float outputs)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))
