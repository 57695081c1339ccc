"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs the oracle-vs-golden pins, the host logic and the C-ABI loader
checks on CPU; `-m gpu` runs the parity tests proper, which call the sm_100a kernels
through the C ABI and compare them with the CPU oracle and the golden fixtures.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "fni8-serve_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libfni8_b200.so")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))

    return load
