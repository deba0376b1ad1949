"""Shared test configuration.

Markers: ``gpu`` tests need a B200 (they call the CUDA path through the C
ABI and compare with the oracle); everything else runs on CPU.  Tolerances
mirror the reference's ``tests/conftest.py:67-96`` (``tol_for``) where the
reference pins a value, and the stricter bars of the build target where it
states one (bit-exact integers and divisions, <= 2 ulp transcendentals,
1e-4 relative error for float reductions and scans, 1e-5 relative
Frobenius error for float32 matmul).
"""

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device")


def tol_for(dtype, category="default"):
    """Tolerances of the reference's conftest (tests/conftest.py:67-96)."""
    dtype = np.dtype(dtype)
    if category == "arithmetic":
        return dict(rtol=1e-2, atol=1e-2) if dtype == np.float16 else dict(rtol=1e-6, atol=1e-4)
    if category == "unary_math":
        return dict(rtol=1e-2, atol=1e-2) if dtype == np.float16 else dict(rtol=1e-5, atol=1e-5)
    if dtype == np.float16:
        return dict(rtol=1e-2, atol=1e-3)
    if dtype in (np.float32, np.complex64):
        return dict(rtol=1e-5, atol=1e-6)
    return dict(rtol=0, atol=0)


@pytest.fixture(autouse=True)
def _reset_config():
    try:
        from macmetalpy_b200._config import get_config
    except Exception:
        yield
        return
    cfg = get_config()
    saved = (cfg.float64_behavior, cfg.warn_on_downcast, cfg.default_float_dtype, cfg.fast_math)
    yield
    cfg.float64_behavior, cfg.warn_on_downcast, cfg.default_float_dtype, cfg.fast_math = saved
