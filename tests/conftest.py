"""Shared test setup: the repository root and the package directory on sys.path, the `gpu` marker, fixtures."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "pyodide-llm_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built libpllm.so")


@pytest.fixture(scope="session")
def golden():
    """The committed known answers (tests/golden/make_golden.py)."""
    with np.load(os.path.join(ROOT, "tests", "golden", "golden.npz")) as z:
        return {k: z[k] for k in z.files}
