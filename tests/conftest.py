import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: CPU test that takes more than a few seconds")


def golden_files(prefix="ref_"):
    return sorted(f for f in os.listdir(GOLDEN) if f.startswith(prefix) and f.endswith(".npz"))


def allclose_report(actual, expected, rtol=1e-5, atol=5e-6):
    """max |a-e| / (atol + rtol |e|); <= 1 means within tolerance."""
    import numpy as np
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    if a.size == 0:
        return 0.0
    return float((np.abs(a - e) / (atol + rtol * np.abs(e))).max())
