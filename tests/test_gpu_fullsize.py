"""Parity at the BASELINE sizes (configs C2-C5), whole arrays: every
element of every C2 op at 2^28 against the oracle, every element of the
2^30 scans against a chunked host prefix (int64 exact, float64 for float32),
every row of the (4096, 65536) axis-1 scan, the C3 reductions at 16384^2
against float64 numpy, every batch of the batched C5 matmul; the two
square C5 matmuls on sampled rows (a float64 16384^3 host product would
take minutes).  Bars: bit-exact for integers and the
division ops, <= 2 ulp for the transcendental, 1e-4 relative for float
reductions and scans, 1e-5 relative Frobenius for float32 matmul."""

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
    for op, fn in ((cp.add, O.add), (cp.floor_divide, O.floor_divide), (cp.remainder, O.mod)):
        np.testing.assert_array_equal(op(A, B).get(), fn(a, b), err_msg=op.__name__)
    lae = cp.logaddexp(A, B).get()
    for lo in range(0, n, 1 << 26):  # float64 reference in chunks (host memory)
        sl = slice(lo, lo + (1 << 26))
        ref = np.logaddexp(a[sl].astype(np.float64), b[sl].astype(np.float64))
        scale = np.maximum(np.abs(ref), np.maximum(np.abs(a[sl]), np.abs(b[sl])).astype(np.float64))
        assert np.max(np.abs(lae[sl] - ref) / np.spacing(scale.astype(np.float32))) <= 2
    del A, B, a, b, lae
    ai = rng.integers(-1000, 1000, n).astype(np.int32)
    bi = (rng.integers(1, 50, n) * rng.choice(np.array([-1, 1], np.int32), n)).astype(np.int32)
    Ai, Bi = cp.array(ai), cp.array(bi)
    for op, fn in ((cp.add, O.add), (cp.floor_divide, O.floor_divide), (cp.remainder, O.mod)):
        np.testing.assert_array_equal(op(Ai, Bi).get(), fn(ai, bi), err_msg=op.__name__ + " int32")


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


def _chunks(Y, n, step=1 << 27):
    """(lo, hi, device chunk read back) over a 1-D device array."""
    for lo in range(0, n, step):
        hi = min(n, lo + step)
        yield lo, hi, Y[lo:hi].get()


def test_c4_scans_2pow30(cp):
    n = 1 << 30
    rng = np.random.default_rng(3)
    x = rng.integers(-100, 101, n, dtype=np.int32)
    Y = cp.cumsum(cp.array(x))
    assert Y.dtype == np.int64
    carry = 0
    for lo, hi, got in _chunks(Y, n):
        want = np.cumsum(x[lo:hi], dtype=np.int64) + carry
        np.testing.assert_array_equal(got, want)
        carry = int(want[-1])
    del Y, x
    xf = rng.uniform(0, 1, n).astype(np.float32)
    Yf = cp.cumsum(cp.array(xf))
    carry = 0.0
    for lo, hi, got in _chunks(Yf, n):
        ref = np.cumsum(xf[lo:hi].astype(np.float64)) + carry
        assert np.max(np.abs(got - ref) / ref) <= 1e-4
        carry = float(ref[-1])
    del Yf, xf
    x2 = rng.standard_normal((4096, 65536), dtype=np.float32)
    Y2 = cp.cumsum(cp.array(x2), axis=1)
    for r0 in range(0, 4096, 512):
        # normwise per row: an N(0,1) row's prefix crosses zero, where an
        # elementwise relative error is not defined by the data
        ref = np.cumsum(x2[r0:r0 + 512].astype(np.float64), axis=1)
        got = Y2[r0:r0 + 512].get()
        err = np.max(np.abs(got - ref), axis=1) / np.max(np.abs(ref), axis=1)
        assert np.max(err) <= 1e-4


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
    for i in range(0, 64, 16):  # every batch, 16 at a time against a float64 product
        r = ba[i:i + 16].astype(np.float64) @ bb[i:i + 16].astype(np.float64)
        err = np.linalg.norm(G[i:i + 16] - r, axis=(1, 2)) / np.linalg.norm(r, axis=(1, 2))
        assert np.max(err) <= 1e-5
    del G, ba, bb
    ha = (rng.standard_normal((8192, 8192), dtype=np.float32) / np.float32(90.5)).astype(np.float16)
    hb = (rng.standard_normal((8192, 8192), dtype=np.float32) / np.float32(90.5)).astype(np.float16)
    H = cp.matmul(cp.array(ha), cp.array(hb))
    assert H.dtype == np.float16
    rows = rng.choice(8192, 32, replace=False)
    r = ha[rows].astype(np.float64) @ hb.astype(np.float64)
    assert np.linalg.norm(H.get()[rows] - r) / np.linalg.norm(r) <= 2e-3
