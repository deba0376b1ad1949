"""Advanced indexing and the indexing routines on the device against the
reference's golden vectors (tests/golden/golden_index_v1.npz) and numpy:
boolean masks (full-shape and leading-dims), integer arrays (negative,
broadcast, adjacent / separated placement, with slices, ints and newaxis),
views as sources and targets, out-of-range IndexError, assignment forms,
take / put modes, nonzero, compress, extract, putmask, place, select,
choose, unravel / ravel_multi_index, fill_diagonal; bit-exact."""

import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

X = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_index_v1.npz"))


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


def test_golden_getitem(cp):
    a, m, i0, i1, i2, v = (X[k] for k in ("a", "m", "i0", "i1", "i2", "v"))
    A, V = cp.array(a), cp.array(v)
    same(A[cp.array(m)], X["get_mask"])
    same(A[cp.array(i0)], X["get_i0"])
    same(A[cp.array(i0[:3]), :, cp.array(i2)], X["get_i0_i2"])
    same(A[1:5, cp.array(i1)], X["get_s_i1"])
    same(A[2, :, cp.array(i2)], X["get_int_arr"])
    same(A[cp.array(i1 % 6), cp.array(i1 % 7)], X["get_i1_i1"])
    same(A[cp.array(m[:, 0, 0])], X["get_mask_rows"])
    same(A[None, cp.array(i0), ::2], X["get_newaxis"])
    same(V[cp.array(np.array([-1, -40, 3, 39]))], X["get_v_neg"])
    # host index objects work the same
    same(A[m], X["get_mask"])
    same(A[list(i0)], X["get_i0"])


def test_golden_setitem(cp):
    a, m, i0 = X["a"], X["m"], X["i0"]
    B = cp.array(a)
    B[cp.array(m)] = -1.0
    same(B, X["set_mask_scalar"])
    B = cp.array(a)
    B[cp.array(i0[:3]), 2] = cp.array(np.arange(24, dtype=np.float32).reshape(3, 8))
    same(B, X["set_i0_row"])
    B = cp.array(a)
    B[:, cp.array(np.array([6, 0])), 1] = 7.0
    same(B, X["set_cols"])


def test_golden_routines(cp):
    a, m, v = X["a"], X["m"], X["v"]
    A, M, V = cp.array(a), cp.array(m), cp.array(v)
    same(cp.take(V, cp.array(np.array([0, 5, 39, -2]))), X["take_v"])
    same(cp.take(A, cp.array(np.array([6, 0, 3])), axis=1), X["take_ax1"])
    same(cp.take(V, cp.array(np.array([40, -41, 100])), mode="wrap"), X["take_wrap"])
    same(cp.take(V, cp.array(np.array([40, -41, 100])), mode="clip"), X["take_clip"])
    same(cp.take_along_axis(A, cp.array(X["ta"]), axis=2), X["take_along"])
    for k, x in enumerate(cp.nonzero(M)):
        same(x, X[f"nonzero_{k}"])
    same(cp.flatnonzero(M), X["flatnonzero"])
    same(cp.argwhere(cp.array(m[0])), X["argwhere"])
    same(cp.compress(cp.array(X["cond"]), A, axis=1), X["compress_ax1"])
    same(cp.extract(M, A), X["extract"])
    P = cp.array(v)
    cp.put(P, cp.array(np.array([0, 3, 39])), cp.array(np.array([100, 200], np.int32)))
    same(P, X["put"])
    P = cp.array(v)
    cp.putmask(P, cp.array(v > 0), cp.array(np.array([7, 8, 9], np.int32)))
    same(P, X["putmask"])


def test_views_and_dtypes(cp):
    rng = np.random.default_rng(3)
    for dt in (np.bool_, np.int16, np.int32, np.int64, np.float16, np.float32, np.float64, np.uint64):
        x = (rng.standard_normal((9, 11, 5)) * 100).astype(dt)
        Xd = cp.array(x)
        view = Xd[1:8:2, ::-1]  # a strided, reversed view as the source
        xv = x[1:8:2, ::-1]
        idx = np.array([3, 0, -2, 3])
        same(view[:, idx], O.getitem(xv, (slice(None), idx)))
        mk = xv > xv.mean() if dt != np.bool_ else xv
        same(view[mk], O.getitem(xv, mk))
        T = cp.array(x)
        T[2:, ::2][np.array([0, -1]), 1] = x[0, 0, 0]  # assignment through a view
        want = x.copy()
        want[2:, ::2][np.array([0, -1]), 1] = x[0, 0, 0]
        same(T, want)


def test_bounds_and_errors(cp):
    A = cp.array(np.arange(20, dtype=np.float32).reshape(4, 5))
    with pytest.raises(IndexError):
        A[cp.array(np.array([0, 4]))]
    with pytest.raises(IndexError):
        A[:, np.array([-6])]
    with pytest.raises(IndexError):
        A[np.ones((3, 5), bool)]
    with pytest.raises(IndexError):
        A[np.array([0.5])]
    with pytest.raises(IndexError):
        cp.take(A, cp.array(np.array([20])))
    same(A[np.zeros((4, 5), bool)], np.zeros(0, np.float32))
    same(A[np.array([], dtype=np.int64)], np.zeros((0, 5), np.float32))


def test_large_mask_and_gather(cp):
    rng = np.random.default_rng(4)
    n = 1 << 22
    x = rng.standard_normal(n).astype(np.float32)
    Xd = cp.array(x)
    m = x > 0.5
    same(Xd[Xd > 0.5], x[m])
    idx = rng.integers(-n, n, 1 << 20)
    same(Xd[cp.array(idx)], x[idx])
    Y = cp.array(x)
    Y[Y < 0] = 0.0
    same(Y, np.where(x < 0, np.float32(0), x))
    Z = cp.array(x)
    sel = rng.choice(n, 1000, replace=False)
    Z[cp.array(sel)] = cp.array(np.arange(1000, dtype=np.float32))
    want = x.copy()
    want[sel] = np.arange(1000, dtype=np.float32)
    same(Z, want)


def test_more_routines(cp):
    rng = np.random.default_rng(5)
    x = rng.integers(-9, 10, (6, 8)).astype(np.int32)
    Xd = cp.array(x)
    P = cp.array(x)
    cp.place(P, cp.array(x > 3), cp.array(np.array([1, 2], np.int32)))
    want = x.copy()
    np.place(want, x > 3, np.array([1, 2], np.int32))
    same(P, want)
    c1, c2 = x > 5, x < -5
    same(cp.select([cp.array(c1), cp.array(c2)], [Xd, Xd * 2], default=-1),
         np.select([c1, c2], [x, x * 2], default=-1))
    ch = rng.integers(0, 3, (6, 8))
    same(cp.choose(cp.array(ch), [Xd, Xd + 1, Xd * 3]), np.choose(ch, [x, x + 1, x * 3]))
    flat = rng.integers(0, 6 * 8 * 7, 100)
    for got, want in zip(cp.unravel_index(cp.array(flat), (6, 8, 7)), np.unravel_index(flat, (6, 8, 7))):
        same(got, want.astype(np.int64))
    r, c = rng.integers(0, 6, 50), rng.integers(0, 8, 50)
    same(cp.ravel_multi_index((cp.array(r), cp.array(c)), (6, 8)), np.ravel_multi_index((r, c), (6, 8)))
    D = cp.array(np.zeros((5, 5), np.float32))
    cp.fill_diagonal(D, 3.0)
    same(D, np.eye(5, dtype=np.float32) * 3)
    E = cp.array(np.zeros((7, 3), np.float32))
    cp.fill_diagonal(E, 1.0, wrap=True)
    e = np.zeros((7, 3), np.float32)
    np.fill_diagonal(e, 1.0, wrap=True)
    same(E, e)
    same(cp.where(cp.array(x > 0))[1], np.where(x > 0)[1])
    ta = rng.integers(0, 8, (6, 2))
    Q = cp.array(x)
    cp.put_along_axis(Q, cp.array(ta), 99, axis=1)
    want = x.copy()
    np.put_along_axis(want, ta, 99, axis=1)
    same(Q, want)
    ix = cp.ix_(cp.array(np.array([0, 5])), cp.array(np.array([1, 2, 7])))
    same(Xd[ix], x[np.ix_([0, 5], [1, 2, 7])])
