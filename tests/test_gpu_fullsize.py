"""Parity at the BASELINE sizes (configs C2-C5), through properties that do
not need the oracle to process the whole array: oracle comparison on
sampled positions or windows, conservation (last prefix == total),
differencing (y[i] - y[i-1] == x[i]), and float64 references on sampled
rows.  Bars: bit-exact for integers and the division ops, <= 2 ulp for the
transcendental, 1e-4 relative for float reductions and scans, 1e-5
relative Frobenius for float32 matmul."""

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    return cp


def test_c2_binary_2pow28(cp):
    n = 1 << 28
    rng = np.random.default_rng(0)
    a = rng.uniform(-1000, 1000, n).astype(np.float32)
    b = (rng.uniform(1, 50, n) * rng.choice(np.array([-1, 1], np.float32), n)).astype(np.float32)
    A, B = cp.array(a), cp.array(b)
    idx = rng.integers(0, n, 1 << 20)
    for got, fn in ((cp.add(A, B), O.add), (cp.floor_divide(A, B), O.floor_divide), (A % B, O.mod)):
        np.testing.assert_array_equal(got.get()[idx], fn(a[idx], b[idx]))
    lae = cp.logaddexp(A, B).get()[idx]
    ref = np.logaddexp(a[idx].astype(np.float64), b[idx].astype(np.float64))
    scale = np.maximum(np.abs(ref), np.maximum(np.abs(a[idx]), np.abs(b[idx])).astype(np.float64))
    assert np.max(np.abs(lae - ref) / np.spacing(scale.astype(np.float32))) <= 2
    del A, B, a, b
    ai = rng.integers(-1000, 1000, n).astype(np.int32)
    bi = (rng.integers(1, 50, n) * rng.choice(np.array([-1, 1], np.int32), n)).astype(np.int32)
    Ai, Bi = cp.array(ai), cp.array(bi)
    for got, fn in ((cp.add(Ai, Bi), O.add), (cp.floor_divide(Ai, Bi), O.floor_divide), (Ai % Bi, O.mod)):
        np.testing.assert_array_equal(got.get()[idx], fn(ai[idx], bi[idx]))


def test_c2_broadcast_add_full(cp):
    rng = np.random.default_rng(1)
    r = rng.standard_normal((8192, 1)).astype(np.float32)
    c = rng.standard_normal((1, 32768)).astype(np.float32)
    np.testing.assert_array_equal((cp.array(r) + cp.array(c)).get(), r + c)


def test_c3_reductions_16384(cp):
    rng = np.random.default_rng(2)
    a = rng.standard_normal((16384, 16384), dtype=np.float32)
    A = cp.array(a)
    a64 = a.astype(np.float64)
    for fn, ref in ((cp.sum, np.sum), (cp.mean, np.mean), (cp.var, np.var)):
        got = float(fn(A).get())
        want = float(ref(a64))
        assert abs(got - want) <= 1e-4 * max(abs(want), 1e-3 * np.abs(a64).sum()), fn.__name__
        for ax in (0, 1):
            g = fn(A, axis=ax).get()
            w = ref(a64, axis=ax)
            floor = 1e-3 * np.abs(a64).mean(axis=ax) * (16384 if fn is cp.sum else 1)
            assert np.max(np.abs(g - w) / np.maximum(np.abs(w), floor)) <= 1e-4, (fn.__name__, ax)
    assert cp.argmax(A) == O.argmax(a)
    np.testing.assert_array_equal(cp.argmax(A, axis=0).get(), O.argmax_axis(a, 0))
    np.testing.assert_array_equal(cp.argmax(A, axis=1).get(), O.argmax_axis(a, 1))
    an = a.copy()
    an.reshape(-1)[rng.choice(an.size, an.size // 100, replace=False)] = np.nan
    An = cp.array(an)
    assert abs(float(cp.nansum(An).get()) - np.nansum(an.astype(np.float64))) <= 1e-4 * np.nansum(np.abs(an))
    nm = np.nanmean(an.astype(np.float64))
    assert abs(float(cp.nanmean(An).get()) - nm) <= 1e-4 * max(abs(nm), 1e-3 * np.nanmean(np.abs(an)))
    del A, An, a64, an
    bi = rng.integers(-100, 101, (16384, 16384)).astype(np.int32)
    assert int(cp.sum(cp.array(bi)).get()) == int(O.reduce_sum(bi))


def test_c4_scans_2pow30(cp):
    n = 1 << 30
    rng = np.random.default_rng(3)
    x = rng.integers(-100, 101, n, dtype=np.int32)
    X = cp.array(x)
    Y = cp.cumsum(X)
    assert Y.dtype == np.int64
    # conservation and differencing on the device, a few windows on the host
    assert int(Y[-1].get()) == int(x.sum(dtype=np.int64))
    d = Y[1:] - Y[:-1]
    assert not bool((d != X[1:]).any().get())
    for s in (0, 4095, 123456789, n - 5000):
        w = Y[s:s + 5000].get()
        base = 0 if s == 0 else int(x[:s].sum(dtype=np.int64))
        np.testing.assert_array_equal(w, base + np.cumsum(x[s:s + 5000], dtype=np.int64))
    del X, Y, d, x
    xf = rng.uniform(0, 1, n).astype(np.float32)
    Yf = cp.cumsum(cp.array(xf))
    for s in (0, 777777, 500000000, n - 4096):
        w = Yf[s:s + 4096].get().astype(np.float64)
        ref = float(xf[:s].astype(np.float64).sum()) + np.cumsum(xf[s:s + 4096].astype(np.float64))
        assert np.max(np.abs(w - ref) / ref) <= 1e-4
    del Yf, xf
    x2 = rng.standard_normal((4096, 65536), dtype=np.float32)
    Y2 = cp.cumsum(cp.array(x2), axis=1)
    for r in (0, 1, 2047, 4095):
        # normwise: an N(0,1) row's prefix crosses zero, where an elementwise
        # relative error is not defined by the data
        ref = np.cumsum(x2[r].astype(np.float64))
        got = Y2[r].get()
        assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) <= 1e-4


def test_c5_matmul_baseline_shapes(cp):
    rng = np.random.default_rng(4)
    n = 16384
    a = (rng.standard_normal((n, n), dtype=np.float32) / np.float32(128))
    b = (rng.standard_normal((n, n), dtype=np.float32) / np.float32(128))
    C = cp.matmul(cp.array(a), cp.array(b))
    rows = rng.choice(n, 48, replace=False)
    ref = a[rows].astype(np.float64) @ b.astype(np.float64)
    got = C.get()[rows]
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-5
    del C, a, b
    ba = (rng.standard_normal((64, 1024, 1024), dtype=np.float32) / np.float32(32))
    bb = (rng.standard_normal((64, 1024, 1024), dtype=np.float32) / np.float32(32))
    G = cp.matmul(cp.array(ba), cp.array(bb)).get()
    for i in (0, 31, 63):
        r = ba[i].astype(np.float64) @ bb[i].astype(np.float64)
        assert np.linalg.norm(G[i] - r) / np.linalg.norm(r) <= 1e-5
    del G, ba, bb
    ha = (rng.standard_normal((8192, 8192), dtype=np.float32) / np.float32(90.5)).astype(np.float16)
    hb = (rng.standard_normal((8192, 8192), dtype=np.float32) / np.float32(90.5)).astype(np.float16)
    H = cp.matmul(cp.array(ha), cp.array(hb))
    assert H.dtype == np.float16
    rows = rng.choice(8192, 32, replace=False)
    r = ha[rows].astype(np.float64) @ hb.astype(np.float64)
    assert np.linalg.norm(H.get()[rows] - r) / np.linalg.norm(r) <= 2e-3
