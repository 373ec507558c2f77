"""Shared fixtures. `-m gpu` tests run the CUDA kernels through the C ABI and compare with
the CPU oracle (oracle/); `-m "not gpu"` tests cover the oracle, host logic and the ABI
surface without a GPU."""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")
    config.addinivalue_line("markers", "slow: full-size cases (seconds of CPU oracle work)")


def load_pkg():
    return importlib.import_module("recursive-routing-racer-rs_b200")


@pytest.fixture(scope="session")
def rrr():
    pkg = load_pkg()
    from importlib import import_module
    import_module("recursive-routing-racer-rs_b200.build").build()
    return pkg


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.build()
    return o


@pytest.fixture(scope="session")
def ctx(rrr):
    c = rrr.Context(0)
    yield c
    code = c.device_error()
    c.close()
    assert code == 0, f"a kernel reported device error code {code}"


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
