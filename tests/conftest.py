"""Shared test setup: the gpu marker, import paths, and the libraries under test.

Markers: `gpu` tests need a CUDA device and call the B200 library through its C ABI; everything else runs on the
CPU (the oracle against the golden vectors, the host logic, the library's exports and refusals)."""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "radiance-exl3_b200"
for p in (str(PKG), str(REPO / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and runs the sm_100a kernels")


@pytest.fixture(scope="session")
def repo():
    return REPO
