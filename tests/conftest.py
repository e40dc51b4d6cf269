"""Shared pytest configuration.

Markers:
  gpu  - needs a CUDA device (B200); run with `pytest -m gpu`.
Everything else runs on a CPU-only machine.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cwlb-spmm_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    """The reference's own code (oracle/_ref); skipped where it was not built."""
    from oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/libcwlbref.so not built (no reference checkout)")
    r = Reference()
    r.set_device()
    return r


@pytest.fixture(scope="session")
def golden_costs():
    with open(os.path.join(GOLDEN, "spmm_costs.txt")) as f:
        return np.array([float(x) for x in f.read().split()[:4]])


def load_npz(name):
    return np.load(os.path.join(GOLDEN, name))
