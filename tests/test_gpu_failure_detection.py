"""Failure detection without a GPU fault: a kernel whose bounded wait runs
out (a flag that nothing sets) reports device error 6 through
mmp_check_device_error / cp.synchronize(), and the context stays usable
for the next kernels (the scan's look-back and the GEMM's mbarrier waits
follow the same rule: bounded, error word, return)."""

import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_context_survives():
    import macmetalpy_b200 as cp
    from macmetalpy_b200 import _cuda_backend as cb

    cp.synchronize()
    polls = ctypes.c_uint(0)
    t0 = time.perf_counter()
    assert cb.lib.mmp_selftest_bounded_wait(200000, ctypes.byref(polls)) == 0  # 0.2 s limit
    assert time.perf_counter() - t0 < 5.0
    assert polls.value > 0
    code = ctypes.c_int(0)
    assert cb.lib.mmp_check_device_error(ctypes.byref(code)) == 0
    assert code.value == 6
    # read once, then cleared
    assert cb.lib.mmp_check_device_error(ctypes.byref(code)) == 0 and code.value == 0
    # the same condition surfaces as an exception from cp.synchronize()
    assert cb.lib.mmp_selftest_bounded_wait(50000, None) == 0
    with pytest.raises(RuntimeError, match="device error code 6"):
        cp.synchronize()
    # the context is still usable
    x = np.arange(1000, dtype=np.float32)
    np.testing.assert_array_equal(cp.cumsum(cp.array(x)).get(), np.cumsum(x))
