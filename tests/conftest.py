"""Shared test setup: markers, import paths, GPU fixtures.

`-m "not gpu"` runs on any host: the oracle against the golden fixtures made
from the reference's own kernels, host logic, and the C ABI's exports.
`-m gpu` runs the CUDA path through the C ABI against the oracle.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "project-obsidian_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path through the C ABI)")


def pytest_collection_modifyitems(config, items):
    # a bound on every test: the device-side waits are bounded (2 s by default),
    # so a test that keeps hitting them fails here instead of running for long
    try:
        import pytest_timeout  # noqa: F401
    except ImportError:
        return
    for item in items:
        if item.get_closest_marker("timeout") is None:
            item.add_marker(pytest.mark.timeout(600))


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device on this host")
    return torch


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    d = os.path.join(ROOT, "tests", "golden")

    def load(name):
        return dict(np.load(os.path.join(d, f"ref_{name}.npz")))

    return load
