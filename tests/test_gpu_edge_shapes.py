"""Edge shapes on the device against numpy (the reference's CPU path):
empty arrays, zero-length axes, 0-d arrays, size-1 dimensions and
reversed views, through elementwise / broadcast ops, reductions, scans,
sort, matmul and indexing.  Values and dtypes exact (float reductions of
empty input are NaN as numpy's)."""

import warnings

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
warnings.simplefilter("ignore", RuntimeWarning)


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    return cp


def same(got, want):
    got = got.get() if hasattr(got, "get") else np.asarray(got)
    want = np.asarray(want)
    assert got.dtype == want.dtype, (got.dtype, want.dtype)
    assert got.shape == want.shape, (got.shape, want.shape)
    np.testing.assert_array_equal(got, want)


def test_empty_elementwise_and_broadcast(cp):
    e = np.zeros(0, np.float32)
    E = cp.array(e)
    same(E + E, e + e)
    same(cp.exp(E), np.exp(e))
    r, c = np.zeros((0, 1), np.float32), np.ones((1, 5), np.float32)
    same(cp.array(r) + cp.array(c), r + c)
    same(cp.where(cp.array(np.zeros(0, bool)), E, 1.0), np.where(np.zeros(0, bool), e, np.float32(1.0)))
    ei = np.zeros((3, 0), np.int32)
    same(cp.floor_divide(cp.array(ei), 7), np.floor_divide(ei, np.int32(7)))


def test_empty_reductions_and_axes(cp):
    e = np.zeros(0, np.float32)
    E = cp.array(e)
    same(cp.sum(E), np.sum(e))
    assert np.isnan(float(cp.mean(E).get())) and np.isnan(float(cp.var(E).get()))
    z = np.zeros((0, 5), np.float32)
    Z = cp.array(z)
    same(cp.sum(Z, axis=0), np.sum(z, axis=0))
    same(cp.sum(Z, axis=1), np.sum(z, axis=1))
    same(cp.prod(Z, axis=0), np.prod(z, axis=0))
    zi = np.zeros((4, 0), np.int32)
    same(cp.sum(cp.array(zi), axis=1), np.sum(zi, axis=1))
    assert cp.count_nonzero(E) == 0
    assert bool(cp.all(E).get()) is True and bool(cp.any(E).get()) is False
    with pytest.raises(ValueError):
        cp.argmax(Z, axis=0)


def test_empty_scans_sort_matmul_indexing(cp):
    ei = np.zeros(0, np.int32)
    same(cp.cumsum(cp.array(ei)), np.cumsum(ei))
    z = np.zeros((3, 0), np.float32)
    same(cp.cumsum(cp.array(z), axis=1), np.cumsum(z, axis=1))
    same(cp.sort(cp.array(ei)), np.sort(ei))
    same(cp.argsort(cp.array(ei)), np.argsort(ei))
    a, b = np.ones((3, 0), np.float32), np.ones((0, 4), np.float32)
    same(cp.matmul(cp.array(a), cp.array(b)), np.matmul(a, b))
    a2 = np.ones((0, 5), np.float32)
    same(cp.matmul(cp.array(a2), cp.array(np.ones((5, 4), np.float32))), np.matmul(a2, np.ones((5, 4), np.float32)))
    m = np.zeros(7, bool)
    x = np.arange(7, dtype=np.float32)
    same(cp.array(x)[cp.array(m)], x[m])
    same(cp.nonzero(cp.array(m))[0], np.nonzero(m)[0])


def test_zero_d(cp):
    a, b = np.float32(2.5), np.float32(-4.0)
    A, B = cp.array(a), cp.array(b)
    assert A.shape == () and (A + B).shape == ()
    same(A + B, np.asarray(a + b))
    same(cp.floor_divide(B, A), np.asarray(np.floor_divide(b, a)))
    same(cp.sum(A), np.asarray(np.sum(a)))
    same(cp.cumsum(A), np.cumsum(a))
    assert cp.argmax(A) == 0
    same(A * cp.array(np.ones((2, 3), np.float32)), a * np.ones((2, 3), np.float32))
    with pytest.raises(np.exceptions.AxisError):
        cp.sort(A)


def test_size_one_dims_and_reversed_views(cp):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 7, 1, 5)).astype(np.float32)
    X = cp.array(x)
    for ax in (None, 0, 1, 2, 3, -1):
        np.testing.assert_allclose(cp.sum(X, axis=ax).get(), np.sum(x.astype(np.float64), axis=ax),
                                   rtol=1e-6, atol=1e-6)
    same(cp.argmax(X, axis=1), np.argmax(x, axis=1).astype(np.int32))
    cs = cp.cumsum(X, axis=1)  # float carries are float64: within the scan bar of the float64 scan
    assert cs.dtype == np.float32 and cs.shape == x.shape
    np.testing.assert_allclose(cs.get(), np.cumsum(x.astype(np.float64), axis=1), rtol=1e-6, atol=1e-6)
    y = rng.integers(-50, 50, (6, 9)).astype(np.int32)
    Y = cp.array(y)
    rv = Y[::-1, ::-2]
    yv = y[::-1, ::-2]
    same(rv + 1, yv + 1)
    same(cp.sum(rv, axis=0), np.sum(yv, axis=0))
    same(cp.cumsum(rv, axis=1), np.cumsum(yv, axis=1))
    same(cp.sort(rv, axis=0), np.sort(yv, axis=0))
    same(rv % 7, yv % np.int32(7))
