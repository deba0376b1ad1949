"""Order statistics, unique, lexsort and partition on the device against
numpy (the reference's CPU path for all of them): median / percentile /
quantile and their nan-versions over dtypes, axes (int, tuple, None),
keepdims, q forms (Python scalar, list, float32 array), NaN and all-NaN
slices; unique with first indices, inverse and counts (NaNs equal), along
an axis; lexsort; the partition contract.  Values and dtypes bit-exact."""

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


def data(shape, dt, seed, nan_frac=0.0):
    rng = np.random.default_rng(seed)
    if np.dtype(dt).kind == "f":
        x = (rng.standard_normal(shape) * 10).astype(dt)
        if nan_frac:
            x[rng.random(shape) < nan_frac] = np.nan
        return x
    if np.dtype(dt) == np.bool_:
        return rng.random(shape) < 0.5
    return rng.integers(-50, 50, shape).astype(dt)


@pytest.mark.parametrize("dt", [np.float32, np.float64, np.float16, np.int32, np.int64, np.bool_])
def test_median(cp, dt):
    for shape in [(1001,), (1000,), (7, 9, 10)]:
        x = data(shape, dt, len(shape) + 3)
        X = cp.array(x)
        axes = [None] + list(range(len(shape))) + ([(0, 2)] if len(shape) == 3 else [])
        for ax in axes:
            same(cp.median(X, axis=ax), np.median(x, axis=ax))
            same(cp.median(X, axis=ax, keepdims=True), np.median(x, axis=ax, keepdims=True))
    if np.dtype(dt).kind == "f":
        x = data((6, 11), dt, 5)
        x[2, 3] = np.nan
        same(cp.median(cp.array(x), axis=1), np.median(x, axis=1))
        same(cp.median(cp.array(x)), np.median(x))


@pytest.mark.parametrize("dt", [np.float32, np.float64, np.int32, np.float16])
def test_percentile_quantile(cp, dt):
    x = data((9, 37), dt, 11)
    X = cp.array(x)
    for q in (0, 100, 50, 37.5, 99.9, [10, 50, 90], np.array([25.0, 75.0], np.float32)):
        for ax in (None, 0, 1):
            same(cp.percentile(X, q, axis=ax), np.percentile(x, q, axis=ax))
    for q in (0.0, 1.0, 0.3, [0.1, 0.7], np.float64(0.25)):
        for ax in (None, 1):
            same(cp.quantile(X, q, axis=ax), np.quantile(x, q, axis=ax))
    same(cp.quantile(X, [0.2, 0.9], axis=1, keepdims=True), np.quantile(x, [0.2, 0.9], axis=1, keepdims=True))
    if np.dtype(dt).kind == "f":
        x[4, 7] = np.nan
        same(cp.percentile(cp.array(x), 40, axis=1), np.percentile(x, 40, axis=1))
    with pytest.raises(ValueError):
        cp.percentile(X, 101)


@pytest.mark.parametrize("dt", [np.float32, np.float64, np.float16])
def test_nan_order_stats(cp, dt):
    x = data((12, 41), dt, 21, nan_frac=0.2)
    x[3] = np.nan            # an all-NaN row
    x[5, 1:] = np.nan        # a single value left
    X = cp.array(x)
    for ax in (None, 0, 1):
        same(cp.nanmedian(X, axis=ax), np.nanmedian(x, axis=ax))
        for q in (0, 50, 12.5, 100, [5, 95]):
            same(cp.nanpercentile(X, q, axis=ax), np.nanpercentile(x, q, axis=ax))
        same(cp.nanquantile(X, 0.6, axis=ax), np.nanquantile(x, 0.6, axis=ax))
    same(cp.nanmedian(X, axis=1, keepdims=True), np.nanmedian(x, axis=1, keepdims=True))
    xi = data((5, 8), np.int32, 3)
    same(cp.nanmedian(cp.array(xi), axis=1), np.nanmedian(xi, axis=1))
    same(cp.nanpercentile(cp.array(xi), 30), np.nanpercentile(xi, 30))


def test_large_median_percentile(cp):
    x = data((1 << 20,), np.float32, 8, nan_frac=0.01)
    X = cp.array(x)
    same(cp.nanmedian(X), np.nanmedian(x))
    same(cp.nanpercentile(X, [1, 50, 99]), np.nanpercentile(x, [1, 50, 99]))
    y = data((512, 2049), np.float32, 9)
    same(cp.median(cp.array(y), axis=1), np.median(y, axis=1))
    same(cp.percentile(cp.array(y), 90, axis=0), np.percentile(y, 90, axis=0))


def test_unique(cp):
    rng = np.random.default_rng(4)
    xi = rng.integers(-20, 20, (30, 40)).astype(np.int32)
    Xi = cp.array(xi)
    for got, want in zip(cp.unique(Xi, return_index=True, return_inverse=True, return_counts=True),
                         np.unique(xi, return_index=True, return_inverse=True, return_counts=True)):
        same(got, want)
    same(cp.unique(Xi), np.unique(xi))
    xf = rng.standard_normal(5000).astype(np.float32).round(1)
    xf[rng.random(5000) < 0.05] = np.nan
    Xf = cp.array(xf)
    for got, want in zip(cp.unique(Xf, return_index=True, return_inverse=True, return_counts=True),
                         np.unique(xf, return_index=True, return_inverse=True, return_counts=True)):
        same(got, want)
    # the reference's unique_* call np.unique (sorting.py:330-366): NaNs
    # merge, unlike numpy's array-API unique_values
    ua = cp.unique_all(Xf)
    wa = np.unique(xf, return_index=True, return_inverse=True, return_counts=True)
    for k, w in zip(("values", "indices", "inverse_indices", "counts"), wa):
        same(getattr(ua, k), w)
    same(cp.unique_counts(Xi).counts, np.unique(xi, return_counts=True)[1])
    same(cp.unique_values(Xf), np.unique(xf))
    same(cp.unique(cp.array(np.zeros(0, np.float32))), np.unique(np.zeros(0, np.float32)))
    r = rng.integers(0, 3, (50, 4)).astype(np.int64)
    for got, want in zip(cp.unique(cp.array(r), axis=0, return_index=True, return_inverse=True,
                                   return_counts=True),
                         np.unique(r, axis=0, return_index=True, return_inverse=True, return_counts=True)):
        same(got, want)
    same(cp.unique(cp.array(r), axis=1), np.unique(r, axis=1))


def test_lexsort_partition(cp):
    rng = np.random.default_rng(6)
    k1 = rng.integers(0, 5, 1000).astype(np.int32)
    k2 = rng.standard_normal(1000).astype(np.float32).round(0)
    k3 = rng.integers(0, 3, 1000).astype(np.int16)
    same(cp.lexsort([cp.array(k1), cp.array(k2), cp.array(k3)]), np.lexsort([k1, k2, k3]))
    same(cp.lexsort((cp.array(k2), cp.array(k1))), np.lexsort((k2, k1)))
    m = rng.integers(0, 4, (6, 50)).astype(np.int32)
    same(cp.lexsort(cp.array(m)), np.lexsort(m))
    x = rng.standard_normal((8, 100)).astype(np.float32)
    X = cp.array(x)
    for kth in (0, 37, 99, -1):
        p = cp.partition(X, kth, axis=1).get()
        w = np.partition(x, kth, axis=1)
        np.testing.assert_array_equal(p[:, kth], w[:, kth])
        k = kth % 100
        assert np.all(p[:, :k] <= p[:, k:k + 1]) and np.all(p[:, k + 1:] >= p[:, k:k + 1])
        ap = cp.argpartition(X, kth, axis=1).get()
        np.testing.assert_array_equal(np.take_along_axis(x, ap, axis=1)[:, kth], w[:, kth])
    with pytest.raises(ValueError):
        cp.partition(X, 100, axis=1)


def test_golden_order(cp):
    """Against the reference's own outputs (tests/golden/golden_order_v1.npz)."""
    import os

    R = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_order_v1.npz"))
    A, AN, AI = cp.array(R["a"]), cp.array(R["an"]), cp.array(R["ai"])
    for ax in (None, 0, 1):
        t = "n" if ax is None else str(ax)
        same(cp.median(A, axis=ax), R[f"median_{t}"])
        same(cp.median(AI, axis=ax), R[f"median_i_{t}"])
        same(cp.percentile(A, 37.5, axis=ax), R[f"pct37_{t}"])
        same(cp.percentile(A, [10, 50, 90], axis=ax), R[f"pct_list_{t}"])
        same(cp.percentile(AI, 30, axis=ax), R[f"pct_i_{t}"])
        same(cp.quantile(A, 0.3, axis=ax), R[f"q03_{t}"])
        same(cp.nanmedian(AN, axis=ax), R[f"nanmedian_{t}"])
        same(cp.nanpercentile(AN, 12.5, axis=ax), R[f"nanpct_{t}"])
        same(cp.nanquantile(AN, 0.6, axis=ax), R[f"nanq_{t}"])
    for name in ("u", "uf"):
        got = cp.unique(cp.array(R[name]), return_index=True, return_inverse=True, return_counts=True)
        for g, k in zip(got, ("", "_index", "_inverse", "_counts")):
            same(g, R[f"unique_{name}{k}"])
    same(cp.lexsort([cp.array(R["k1"]), cp.array(R["k2"])]), R["lexsort"])
