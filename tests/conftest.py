"""Shared test setup: the `gpu` marker, import paths and golden-file access."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", os.path.join("tests", "golden"), "voxtral.c_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_golden(name):
    return np.load(os.path.join(ROOT, "tests", "golden", name + ".npz"))


def unpack(g, prefix):
    """(indices, values, full-norm, size) of a packed golden output."""
    return g[prefix + "_idx"], g[prefix + "_val"], float(g[prefix + "_norm"]), int(g[prefix + "_size"])


@pytest.fixture(scope="session")
def golden():
    return load_golden
