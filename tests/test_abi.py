"""The C-ABI library loads on a host without a GPU and exports exactly the
entry points include/mmp_cuda.h declares (no compute calls here)."""

import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    names = set()
    for fn in os.listdir(os.path.join(REPO, "include")):
        if fn.endswith(".h"):
            txt = open(os.path.join(REPO, "include", fn)).read()
            txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
            names |= set(re.findall(r"\b(mmp_[a-z0-9_]+)\s*\(", txt))
    return names


def test_library_exports_header_symbols():
    from macmetalpy_b200 import _cuda_backend as cb
    lib = ctypes.CDLL(cb.LIB_PATH)
    declared = header_functions()
    assert len(declared) >= 25
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from macmetalpy_b200 import _cuda_backend as cb
    assert set(cb.SIGNATURES) == header_functions()


def test_abi_version_and_error_without_device():
    from macmetalpy_b200 import _cuda_backend as cb
    assert cb.lib.mmp_abi_version() == 1
    n = ctypes.c_int(-1)
    rc = cb.lib.mmp_device_count(ctypes.byref(n))
    if rc != 0:  # no driver / GPU on this host: a clean error, not a crash
        assert n.value == 0
        assert cb.lib.mmp_last_error()


def test_argument_checks_fail_cleanly():
    from macmetalpy_b200 import _cuda_backend as cb
    assert cb.lib.mmp_reduce(0, 10, None, -1, 10, None, 0.0, None) == -2
    assert b"negative" in cb.lib.mmp_last_error()
    assert cb.lib.mmp_scan(0, 5, None, 7, None, -1, 1, 1, None) == -2
    assert cb.lib.mmp_gemm(10, 0, 1, -1, 1, 1, None, 1, 0, None, 1, 0, None, 1, 0) == -2
    assert cb.lib.mmp_reduce_axis(0, 10, None, 1, 0, 1, 10, ctypes.c_void_p(16), 0.0) == -2
    assert cb.lib.mmp_sort(10, None, None, None, 1, -1) == -2
    assert cb.lib.mmp_sort(10, ctypes.c_void_p(16), None, None, 1, 8) == -2  # no output
    assert cb.lib.mmp_sort(10, ctypes.c_void_p(16), ctypes.c_void_p(16), None, 1 << 20, 1 << 20) == -2
    assert b"2^32" in cb.lib.mmp_last_error()
    assert cb.lib.mmp_searchsorted(10, None, -1, None, 1, 0, None, None) == -2
    assert cb.lib.mmp_searchsorted(10, ctypes.c_void_p(16), 4, ctypes.c_void_p(16), 1, 2, None,
                                   ctypes.c_void_p(16)) == -2
    assert cb.lib.mmp_gather(10, None, 4, None, -1, None) == -2
    assert cb.lib.mmp_scatter(10, None, -1, None, 1, None) == -2
    assert cb.lib.mmp_compact_indices(None, None, -1, 0, None) == -2
    assert cb.lib.mmp_stream_create(None) == -2
    assert cb.lib.mmp_stream_wait_event(None, None) == -2
    assert cb.lib.mmp_event_record_on(None, None) == -2
    assert cb.lib.mmp_h2d_async(None, None, 16, None) == -2
    assert cb.lib.mmp_selftest_bounded_wait(0, None) == -2


def test_distributed_entry_points_fail_cleanly_without_a_communicator():
    """The partial / merge / collective entry points reject bad arguments and
    report a missing communicator with MMP_E_COMM, without a GPU."""
    from macmetalpy_b200 import _cuda_backend as cb
    assert cb.lib.mmp_reduce_partial(0, 10, None, -1, 0, ctypes.c_void_p(64)) == -2
    assert cb.lib.mmp_reduce_partial(0, 10, ctypes.c_void_p(64), 4, 0, None) == -2
    assert cb.lib.mmp_merge_partials(0, 10, None, -1, 11, ctypes.c_void_p(64), 0.0, None) == -2
    assert cb.lib.mmp_merge_partials(0, 10, ctypes.c_void_p(64), 2, 99, ctypes.c_void_p(64), 0.0, None) == -2
    assert cb.lib.mmp_reduce_allranks(0, 10, None, -1, 0, 11, ctypes.c_void_p(64), 0.0) == -2
    assert cb.lib.mmp_comm_init(0, 0, None, 1.0) == -2
    assert cb.lib.mmp_comm_init(2, 2, ctypes.c_void_p(64), 1.0) == -2
    assert cb.lib.mmp_comm_unique_id(None) == -2
    # no communicator (and, here, no device): a clean error code, no crash
    for rc in (cb.lib.mmp_allreduce(ctypes.c_void_p(64), ctypes.c_void_p(64), 1, 10, 0),
               cb.lib.mmp_allgather(ctypes.c_void_p(64), ctypes.c_void_p(64), 1, 10),
               cb.lib.mmp_broadcast(ctypes.c_void_p(64), ctypes.c_void_p(64), 1, 10, 0),
               cb.lib.mmp_comm_peer_init(), cb.lib.mmp_comm_synchronize(0.1)):
        assert rc in (-2, -6), rc
