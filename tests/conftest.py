"""Shared pytest set-up.

`-m "not gpu"` runs the oracle checks against the reference's golden vectors,
the host-side logic and the library-load/export checks; `-m gpu` runs the
parity tests, which call the CUDA library through its C ABI and compare with
the CPU oracle.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "unlimited-ocr-kernel_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: full-size configuration (seconds of oracle time)")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "quantize_golden.npz"))


@pytest.fixture(scope="session")
def ctx():
    import uocr_q8

    c = uocr_q8.GpuContext(0)
    yield c
    c.close()

