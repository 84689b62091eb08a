"""Shared test setup.

`-m "not gpu"` tests run anywhere (oracle vs golden fixtures, the C ABI's
host-side behaviour, multi-rank host logic on gloo).  `-m gpu` tests need a
B200 and compare the CUDA kernels, called through the C ABI, with the oracle.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Build the library and the oracle once if this tree has not been built yet.
if not os.path.exists(os.path.join(ROOT, "pax_b200", "libpax_b200.so")):
    from pax_b200 import build as _build  # noqa: E402

    _build.build()
if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
    import oracle as _oracle  # noqa: E402

    _oracle.build()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")
    config.addinivalue_line("markers", "slow: large problem sizes")


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    if not gpu_available():
        pytest.skip("no sm_100 GPU")
    import torch

    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


@pytest.fixture
def rng():
    return np.random.default_rng(0x5EED)
