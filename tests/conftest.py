"""Shared test setup: the `gpu` marker, import paths and common fixtures.

Tests marked `gpu` need an sm_100 GPU and the libraries in build/; everything
else runs on a CPU-only machine.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fmha-bwd-gfx1100_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def golden_names():
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))


def load_golden(name):
    import numpy as np

    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: (z[k].item() if z[k].ndim == 0 else z[k]) for k in z.files}


@pytest.fixture(scope="session")
def oracle_built():
    from oracle import oracle as O

    if not os.path.exists(O.ORACLE_SO):
        O.build()
    return O
