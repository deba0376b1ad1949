"""mmp_scan_noalloc: the allocation-free scan, through the C ABI.

This entry point exists for callers that cannot have the library allocate
device memory during a call -- a host framework that keeps nearly all of
HBM in its own pool and passes only its input and output buffers, or code
that runs while that framework holds its allocator lock.  It keeps its
look-back state in a fixed array inside the library instead of scratch
from the memory pool.  Here it must give the same results as mmp_scan on
two calls in a row (the second call reuses the array the first one left
behind), allocate nothing -- the device's default memory pool, which every
library allocation draws from, holds the same number of bytes before and
after a call whose shape is larger than any scan made before it, so the
library's growable look-back state would have had to grow -- and refuse a
scan larger than its fixed array.

The file sorts last so that a run stopping at its first failure has run
every other test before this one."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MMP_INT32, MMP_INT64, MMP_FLOAT32 = 5, 7, 10


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    cp.synchronize()  # initialises the device (mmp_init) before the first call
    return cp


def _scan(lib, fn, x, y, out_code, rows, k):
    rc = fn(0, _code(x), ctypes.c_void_p(x.data_ptr), out_code, ctypes.c_void_p(y.data_ptr), rows, k, 1, None)
    if rc != 0:
        raise RuntimeError(lib.mmp_last_error().decode())


def _code(a):
    return {np.dtype(np.int32): MMP_INT32, np.dtype(np.float32): MMP_FLOAT32}[a.dtype]


@pytest.mark.parametrize("rows,k", [(1, (1 << 22) + 13), (6, 70000)])
def test_noalloc_scan_matches_mmp_scan_twice(cp, rows, k):
    from macmetalpy_b200 import _cuda_backend as cb

    rng = np.random.default_rng(rows)
    xi = cp.array(rng.integers(-100, 101, (rows, k)).astype(np.int32))
    xf = cp.array(rng.uniform(0, 1, (rows, k)).astype(np.float32))
    ref_i = cp.empty((rows, k), dtype=np.int64)
    ref_f = cp.empty((rows, k), dtype=np.float32)
    _scan(cb.lib, cb.lib.mmp_scan, xi, ref_i, MMP_INT64, rows, k)
    _scan(cb.lib, cb.lib.mmp_scan, xf, ref_f, MMP_FLOAT32, rows, k)
    want_i, want_f = ref_i.get(), ref_f.get()
    for _ in range(2):  # the second call starts from the state the first one left
        got_i = cp.empty((rows, k), dtype=np.int64)
        got_f = cp.empty((rows, k), dtype=np.float32)
        _scan(cb.lib, cb.lib.mmp_scan_noalloc, xi, got_i, MMP_INT64, rows, k)
        _scan(cb.lib, cb.lib.mmp_scan_noalloc, xf, got_f, MMP_FLOAT32, rows, k)
        np.testing.assert_array_equal(got_i.get(), want_i)
        g = got_f.get()
        assert np.max(np.abs(g.astype(np.float64) - want_f) / np.maximum(np.abs(want_f), 1e-6)) <= 1e-4
    cp.synchronize()


def test_noalloc_scan_rejects_more_than_its_array(cp):
    from macmetalpy_b200 import _cuda_backend as cb

    x = cp.zeros((16,), dtype=np.int32)
    y = cp.zeros((16,), dtype=np.int64)
    too_long = 1 << 40  # far more tiles than MMP_NOALLOC_SCAN_TILES, whatever the tile size
    # refused on the host before any launch, so the small buffers are never read
    rc = cb.lib.mmp_scan_noalloc(0, MMP_INT32, ctypes.c_void_p(x.data_ptr), MMP_INT64, ctypes.c_void_p(y.data_ptr),
                                 1, too_long, 1, None)
    assert rc == -2
    assert b"exceed" in cb.lib.mmp_last_error()


def _pool_used_bytes():
    """Bytes in use in the current device's default memory pool (the pool
    every allocation of the library comes from), through the driver API."""
    from cuda.bindings import driver as drv

    err, dev = drv.cuCtxGetDevice()
    assert err == drv.CUresult.CUDA_SUCCESS
    err, pool = drv.cuDeviceGetDefaultMemPool(dev)
    assert err == drv.CUresult.CUDA_SUCCESS
    err, used = drv.cuMemPoolGetAttribute(pool, drv.CUmemPool_attribute.CU_MEMPOOL_ATTR_USED_MEM_CURRENT)
    assert err == drv.CUresult.CUDA_SUCCESS
    return int(used)


def test_noalloc_scan_allocates_nothing(cp):
    from macmetalpy_b200 import _cuda_backend as cb

    # 25 x 2048 = 51200 tiles of 4096: beyond the look-back state any scan of
    # this test suite leaves behind, within the fixed array (209715 tiles)
    rows, k = 25, 1 << 23
    rng = np.random.default_rng(9)
    x = cp.array(rng.integers(-100, 101, (rows, k)).astype(np.int32))
    y = cp.empty((rows, k), dtype=np.int64)
    _scan(cb.lib, cb.lib.mmp_scan_noalloc, x, y, MMP_INT64, 1, 4 * 4096)  # first call on the device
    cp.synchronize()
    before = _pool_used_bytes()
    _scan(cb.lib, cb.lib.mmp_scan_noalloc, x, y, MMP_INT64, rows, k)
    cp.synchronize()
    assert _pool_used_bytes() == before
    got = y.get()
    np.testing.assert_array_equal(got, np.cumsum(x.get(), axis=1, dtype=np.int64))

