"""Reductions vs the oracle: full / per-axis / keepdims / ddof, integer
sums bit-exact, argmax ties and NaN, nan-reductions, fused (lazy)
reductions, sizes across block and grid boundaries."""

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SIZES = [1, 2, 7, 31, 32, 33, 255, 1024, 1025, 8191, 65537, 1 << 20, (1 << 22) + 5]


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    return cp


def relerr(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-6)))


@pytest.mark.parametrize("n", SIZES)
def test_full_f32(cp, n):
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32) + 0.5
    X = cp.array(x)
    assert relerr(cp.sum(X).get(), O.sum_f64(x)) <= 1e-4
    assert relerr(cp.mean(X).get(), O.mean_f64(x)) <= 1e-4
    if n > 1:
        assert relerr(cp.var(X).get(), O.var_f64(x)) <= 1e-4
        assert relerr(cp.std(X, ddof=1).get(), np.std(x.astype(np.float64), ddof=1)) <= 1e-4
    assert cp.argmax(X) == O.argmax(x)
    assert cp.argmin(X) == int(np.argmin(x))
    assert float(cp.max(X).get()) == x.max()
    assert float(cp.min(X).get()) == x.min()


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("dtype", [np.int32, np.int16, np.uint32, np.int64, np.bool_])
def test_full_int_exact(cp, n, dtype):
    rng = np.random.default_rng(n + 1)
    x = rng.integers(-100, 101, n).astype(dtype) if dtype != np.bool_ else rng.integers(0, 2, n).astype(bool)
    got = cp.sum(cp.array(x))
    want = O.reduce_sum(x)
    assert got.dtype == want.dtype
    assert got.get() == want


def test_var_large_mean(cp):
    x = (np.random.default_rng(1).standard_normal(1 << 18) + 1e4).astype(np.float32)
    assert relerr(cp.var(cp.array(x)).get(), O.var_f64(x)) <= 1e-4


@pytest.mark.parametrize("shape", [(64, 96), (3, 5), (1000, 3), (3, 1000), (257, 4100), (2, 1 << 17), (16384, 7)])
@pytest.mark.parametrize("axis", [0, 1])
def test_axis_f32(cp, shape, axis):
    a = np.random.default_rng(sum(shape)).standard_normal(shape).astype(np.float32)
    A = cp.array(a)
    # relative to max(|ref|, 1e-3 * mean|x| * k): a sum of zero-mean data may
    # cancel to ~0, where a relative error is not defined by the data
    absmean = O.mean_f64(np.abs(a), axis=axis)
    k = a.shape[axis]
    for fn, ref, fl in ((cp.sum, O.sum_f64, absmean * k), (cp.mean, O.mean_f64, absmean),
                        (cp.var, O.var_f64, absmean ** 2)):
        got = fn(A, axis=axis)
        want = ref(a, axis=axis)
        assert got.shape == want.shape
        assert np.max(np.abs(got.get() - want) / np.maximum(np.abs(want), 1e-3 * fl)) <= 1e-4, fn.__name__
    am = cp.argmax(A, axis=axis)
    assert am.dtype == np.int32
    np.testing.assert_array_equal(am.get(), O.argmax_axis(a, axis))
    np.testing.assert_array_equal(cp.argmin(A, axis=axis).get(), np.argmin(a, axis=axis).astype(np.int32))
    np.testing.assert_array_equal(cp.max(A, axis=axis).get(), a.max(axis=axis))


def test_axis_int_exact_and_3d(cp):
    a = np.random.default_rng(2).integers(-100, 101, (6, 70, 33)).astype(np.int32)
    A = cp.array(a)
    for ax in (0, 1, 2, (0, 2), (1, 2), None):
        got = cp.sum(A, axis=ax)
        want = np.sum(a, axis=ax)
        assert got.dtype == want.dtype
        np.testing.assert_array_equal(np.asarray(got.get()), want)
    np.testing.assert_array_equal(cp.sum(A, axis=1, keepdims=True).get(), a.sum(axis=1, keepdims=True))


def test_argmax_ties_and_nan(cp):
    a = np.array([1, 5, 5, 2, 5], np.float32)
    assert cp.argmax(cp.array(a)) == 1
    b = np.array([1, np.nan, 7, np.nan], np.float32)
    assert cp.argmax(cp.array(b)) == 1
    assert cp.argmin(cp.array(b)) == 1
    big = np.zeros(1 << 20, np.float32)
    big[777777] = np.nan
    big[12345] = np.nan
    assert cp.argmax(cp.array(big)) == 12345
    m = np.zeros((4, 300), np.float32)
    m[2, 17] = 9
    m[2, 200] = 9
    m[1, 5] = np.nan
    np.testing.assert_array_equal(cp.argmax(cp.array(m), axis=1).get(), O.argmax_axis(m, 1))
    np.testing.assert_array_equal(cp.argmax(cp.array(m), axis=0).get(), O.argmax_axis(m, 0))


# Arrays this large take the vector loop that defers the first-occurrence
# search to after the loop: ties between loop steps of different threads,
# all-equal data, several NaNs, many tied extremes, a fused producer.
def test_argmax_large_ties_and_nan(cp):
    n = (1 << 24) + 12
    x = np.zeros(n, np.float32)
    assert cp.argmax(cp.array(x)) == 0 and cp.argmin(cp.array(x)) == 0
    x[[5_000_001, 3_000_017, 9_999_999]] = 7.0
    assert cp.argmax(cp.array(x)) == 3_000_017
    x[[8_000_003, 4_100_000]] = np.nan
    X = cp.array(x)
    assert cp.argmax(X) == 4_100_000 and cp.argmin(X) == 4_100_000
    r = np.random.default_rng(5).integers(-50, 50, n).astype(np.float32)
    R = cp.array(r)
    assert cp.argmax(R) == int(np.argmax(r)) and cp.argmin(R) == int(np.argmin(r))
    assert cp.argmax(-R) == int(np.argmax(-r))
    h = r.astype(np.float16)
    assert cp.argmax(cp.array(h)) == int(np.argmax(h)) and cp.argmin(cp.array(h)) == int(np.argmin(h))
    # rows: ties across the row threads' vectors, and a NaN
    m = np.random.default_rng(6).integers(-20, 20, (64, 65536)).astype(np.float32)
    m[3, 40000] = np.nan
    np.testing.assert_array_equal(cp.argmax(cp.array(m), axis=1).get(), O.argmax_axis(m, 1))
    np.testing.assert_array_equal(cp.argmin(cp.array(m), axis=1).get(), np.argmin(m, axis=1).astype(np.int32))
    # columns (axis 0): four rows folded at once; tied extremes, NaNs, float16
    c = np.random.default_rng(7).integers(-10, 10, (4099, 300)).astype(np.float32)
    c[[5, 2000, 4000], [3, 3, 3]] = np.nan
    c[4098, 10] = np.nan
    c[:, 20] = 1.0
    for arr in (c, c.astype(np.float16)):
        C = cp.array(arr)
        np.testing.assert_array_equal(cp.argmax(C, axis=0).get(), O.argmax_axis(arr, 0))
        np.testing.assert_array_equal(cp.argmin(C, axis=0).get(), np.argmin(arr, axis=0).astype(np.int32))


def test_nan_reductions(cp):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((300, 500)).astype(np.float32)
    a.reshape(-1)[rng.choice(a.size, a.size // 100, replace=False)] = np.nan
    a[7, :] = np.nan
    A = cp.array(a)
    assert relerr(cp.nansum(A).get(), np.nansum(a.astype(np.float64))) <= 1e-4
    assert relerr(cp.nanmean(A).get(), np.nanmean(a.astype(np.float64))) <= 1e-4
    assert np.isnan(cp.sum(A).get())
    got = cp.nanmean(A, axis=1).get()
    want = O.nanmean(a.astype(np.float64), axis=1)
    assert np.isnan(got[7]) and np.isnan(want[7])
    ok = ~np.isnan(want)
    assert np.max(np.abs(got[ok] - want[ok]) / np.maximum(np.abs(want[ok]), 1e-3)) <= 1e-4
    np.testing.assert_array_equal(cp.nanmax(A, axis=0).get(), np.nanmax(a, axis=0))
    assert float(cp.nanmin(A).get()) == np.nanmin(a)


def test_fused_reductions_match_materialised(cp):
    x = np.random.default_rng(4).standard_normal(1 << 20).astype(np.float32)
    X = cp.array(x)
    x64 = x.astype(np.float64)
    y64 = np.sqrt(np.abs(x64)) + np.exp(-(x64 * x64))
    y = cp.sqrt(cp.abs(X)) + cp.exp(-X ** 2)
    assert relerr(cp.sum(y).get(), y64.sum()) <= 1e-4
    assert relerr(cp.mean(y).get(), y64.mean()) <= 1e-4
    assert relerr(cp.var(y).get(), y64.var()) <= 1e-4
    y2 = (cp.sqrt(cp.abs(X)) + cp.exp(-X ** 2)).reshape(1024, 1024)
    Y = y2.copy()
    for ax in (0, 1):
        lazy = (cp.sqrt(cp.abs(X)) + cp.exp(-X ** 2)).reshape(1024, 1024)
        np.testing.assert_allclose(cp.sum(lazy, axis=ax).get(), cp.sum(Y, axis=ax).get(), rtol=1e-6)
    d = cp.dot(X, X)
    assert relerr(d.get(), x64 @ x64) <= 1e-4


def test_empty_and_errors(cp):
    e = cp.array(np.zeros(0, np.float32))
    assert float(cp.sum(e).get()) == 0.0
    with pytest.raises(ValueError):
        cp.max(e)
    with pytest.raises(ValueError):
        cp.argmax(e)


def test_lazy_full_reduction_paths(cp):
    """The short path for a lazy expression reduced to one value and the
    general path agree: out=, the nan-kinds folded to plain kinds on an
    integer expression, result dtypes, an empty lazy input, a repeated
    expression (launch template) with new operands, and keepdims (general
    path) on the same expression."""
    rng = np.random.default_rng(21)
    x = rng.standard_normal(100003).astype(np.float32)
    X = cp.array(x)
    ref = np.sqrt(np.abs(x.astype(np.float64))) + np.exp(-(x.astype(np.float64) ** 2))
    o = cp.empty((), dtype=np.float32)
    r = cp.sum(cp.sqrt(cp.abs(X)) + cp.exp(-X ** 2), out=o)
    assert r is o
    assert relerr(o.get(), ref.sum()) <= 1e-5
    k = cp.sum(cp.sqrt(cp.abs(X)) + cp.exp(-X ** 2), keepdims=True)
    assert k.shape == (1,) and relerr(k.get()[0], ref.sum()) <= 1e-5
    m = cp.mean(cp.sqrt(cp.abs(X)) + cp.exp(-X ** 2))
    assert m.dtype == np.float32 and relerr(m.get(), ref.mean()) <= 1e-5
    xi = rng.integers(-50, 51, 77777).astype(np.int32)
    XI = cp.array(xi)
    s = cp.nansum(XI * 3 + 1)  # no NaN in integers: nansum is sum, int64
    assert s.dtype == np.int64 and int(s.get()) == int((xi.astype(np.int64) * 3 + 1).sum())
    mx = cp.nanmax(XI - 7)
    assert int(mx.get()) == int(xi.max()) - 7
    e = cp.array(np.zeros(0, np.float32))
    assert float(cp.sum(e + 1).get()) == 0.0
    with pytest.raises(ValueError):
        cp.max(e + 1)
    # the same expression again over new arrays: the cached launch takes the
    # new pointers
    for seed in (1, 2):
        y = np.random.default_rng(seed).standard_normal(4096).astype(np.float32)
        Y = cp.array(y)
        got = cp.sum(cp.sqrt(cp.abs(Y)) + cp.exp(-Y ** 2)).get()
        want = (np.sqrt(np.abs(y.astype(np.float64))) + np.exp(-(y.astype(np.float64) ** 2))).sum()
        assert relerr(got, want) <= 1e-5
