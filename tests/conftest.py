"""Shared test setup: import paths, the `gpu` marker and common fixtures."""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PACKAGE = ROOT / "sam.cpp_b200"
for p in (ROOT, PACKAGE):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libsamq.so")


def load_golden(name):
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.lib()
    return o
