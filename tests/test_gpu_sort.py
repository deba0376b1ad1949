"""Device radix sort, argsort and searchsorted against the reference's golden
vectors (tests/golden/golden_sort_v1.npz) and the oracle: bit-exact values
(NaN last, equal_nan comparison), stable int64 argsort (numpy
kind="stable"), every stored dtype, rows / axis=0 / axis=None, ragged
tiles, skipped radix passes (narrow value ranges in wide types), and
searchsorted left / right / sorter with NaN queries."""

import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

S = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_sort_v1.npz"))


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


def test_golden_sort(cp):
    for k in ("f", "i", "d", "h"):
        same(cp.sort(cp.array(S[k])), S[f"sort_{k}"])
    M = cp.array(S["m"])
    same(cp.sort(M, axis=0), S["sort_m_ax0"])
    same(cp.sort(M, axis=1), S["sort_m_ax1"])
    same(cp.sort(M, axis=None), S["sort_m_none"])


def test_golden_argsort(cp):
    same(cp.argsort(cp.array(S["u"])), S["argsort_u"])
    M = cp.array(S["m"])
    same(cp.argsort(M, axis=0), S["argsort_m_ax0"])
    same(cp.argsort(M, axis=1), S["argsort_m_ax1"])


def test_golden_searchsorted(cp):
    SF, Q = cp.array(np.sort(S["f"])), cp.array(S["q"])
    same(cp.searchsorted(SF, Q), S["ss_left"])
    same(cp.searchsorted(SF, Q, side="right"), S["ss_right"])
    SI, QI = cp.array(np.sort(S["i"])), cp.array(S["qi"])
    same(cp.searchsorted(SI, QI), S["ss_i_left"])
    same(cp.searchsorted(SI, QI, side="right"), S["ss_i_right"])
    same(cp.searchsorted(cp.array(S["perm_f"]), Q, sorter=cp.array(S["sorter"])), S["ss_sorter"])
    with pytest.raises(ValueError):
        cp.searchsorted(SF, Q, sorter=cp.array(np.full(S["f"].size, 10 ** 6)))


def _data(dt, n, rng):
    dt = np.dtype(dt)
    if dt == np.bool_:
        return rng.random(n) < 0.5
    if dt.kind in "iu":
        info = np.iinfo(dt)
        return rng.integers(info.min, info.max, n, dtype=dt, endpoint=True)
    x = rng.standard_normal(n).astype(dt)
    x[rng.random(n) < 0.01] = np.nan
    x[rng.random(n) < 0.01] = -np.inf
    x[rng.random(n) < 0.01] = 0.0
    x[rng.random(n) < 0.01] = -0.0
    return x


@pytest.mark.parametrize("dt", [np.bool_, np.int16, np.uint16, np.int32, np.uint32, np.int64, np.uint64,
                                np.float16, np.float32, np.float64])
@pytest.mark.parametrize("n", [1, 7, 4096, 4097, 100003])
def test_dtypes_and_sizes(cp, dt, n):
    rng = np.random.default_rng(n)
    x = _data(dt, n, rng)
    X = cp.array(x)
    same(cp.sort(X), O.sort(x))
    same(cp.argsort(X), O.argsort(x))


def test_rows_axes_and_ties(cp):
    rng = np.random.default_rng(1)
    x = rng.integers(-3, 4, (300, 1001)).astype(np.int32)  # many ties per row
    X = cp.array(x)
    same(cp.sort(X), O.sort(x))
    same(cp.argsort(X), O.argsort(x))
    same(cp.argsort(X, axis=0), O.argsort(x, axis=0))
    same(cp.sort(X, axis=None), O.sort(x, axis=None))
    y = rng.standard_normal((4, 5, 6)).astype(np.float32)
    Y = cp.array(y)
    for ax in (0, 1, 2, -1):
        same(cp.sort(Y, axis=ax), O.sort(y, axis=ax))
        same(cp.argsort(Y, axis=ax), O.argsort(y, axis=ax))
    z = rng.standard_normal((70000, 3)).astype(np.float32)  # many short rows (3 row-id passes)
    same(cp.argsort(cp.array(z)), O.argsort(z))
    Z = cp.array(z.copy())
    Z.sort(axis=0)
    same(Z, O.sort(z, axis=0))


def test_narrow_ranges_skip_passes(cp):
    rng = np.random.default_rng(2)
    for dt in (np.int64, np.uint64, np.int32):
        x = rng.integers(0, 200, 300000).astype(dt)  # only the low byte varies
        same(cp.sort(cp.array(x)), O.sort(x))
        same(cp.argsort(cp.array(x)), O.argsort(x))
    c = np.full(5000, 7, np.int32)  # every pass trivial
    same(cp.argsort(cp.array(c)), np.arange(5000))


def test_large_sort(cp):
    rng = np.random.default_rng(3)
    n = (1 << 24) + 123
    x = rng.standard_normal(n).astype(np.float32)
    X = cp.array(x)
    s = cp.sort(X).get()
    np.testing.assert_array_equal(s, np.sort(x))
    i = cp.argsort(X).get()
    np.testing.assert_array_equal(i, np.argsort(x, kind="stable"))


def test_searchsorted_large_and_nan(cp):
    rng = np.random.default_rng(4)
    a = np.sort(rng.standard_normal(1 << 20).astype(np.float32))
    a[-100:] = np.nan
    v = rng.standard_normal(1 << 18).astype(np.float32)
    v[::97] = np.nan
    A, V = cp.array(a), cp.array(v)
    same(cp.searchsorted(A, V), O.searchsorted(a, v))
    same(cp.searchsorted(A, V, side="right"), O.searchsorted(a, v, side="right"))
    ai = np.sort(rng.integers(-50, 50, 10000)).astype(np.int64)
    same(cp.searchsorted(cp.array(ai), cp.array(np.arange(-60, 60))), O.searchsorted(ai, np.arange(-60, 60)))
    same(cp.searchsorted(cp.array(ai), 3.5), O.searchsorted(ai, 3.5))
    assert cp.searchsorted(cp.array(ai[:0]), cp.array([1, 2])).get().tolist() == [0, 0]
