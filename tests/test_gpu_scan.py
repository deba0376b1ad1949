"""cumsum / cumprod vs the oracle: int32 -> int64 bit-exact across tile
boundaries (4096-element tiles), float32 within 1e-4 of the float64 scan,
row (axis=-1) and column (axis=0) scans, the look-back kernel and the
reduce-then-scan path for long rows, carry-in, back-to-back long scans."""

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SIZES = [1, 2, 31, 1023, 1024, 1025, 4095, 4096, 4097, 3 * 4096 + 5, 40000, (1 << 20) + 7, 1 << 22]


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    return cp


def scan_err(got, ref, x):
    scale = np.cumsum(np.abs(np.asarray(x, np.float64)), axis=-1) * 1e-7 + 1e-30
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref) / np.maximum(np.abs(ref), scale)))


@pytest.mark.parametrize("n", SIZES)
def test_int32_cumsum_exact(cp, n):
    x = np.random.default_rng(n).integers(-100, 101, n).astype(np.int32)
    got = cp.cumsum(cp.array(x))
    want = O.cumsum(x)
    assert got.dtype == np.int64
    np.testing.assert_array_equal(got.get(), want)


@pytest.mark.parametrize("n", SIZES)
def test_f32_cumsum(cp, n):
    x = np.random.default_rng(n + 1).uniform(0, 1, n).astype(np.float32)
    got = cp.cumsum(cp.array(x)).get()
    assert got.dtype == np.float32
    assert scan_err(got, O.cumsum_f64(x), x) <= 1e-4


@pytest.mark.parametrize("shape", [(16, 512), (3, 10000), (4, 65536), (1000, 7), (5, 4096), (2, 4097)])
def test_rows_axis1(cp, shape):
    x = np.random.default_rng(sum(shape)).standard_normal(shape).astype(np.float32)
    got = cp.cumsum(cp.array(x), axis=1).get()
    ref = O.cumsum_f64(x, axis=1)
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) <= 1e-4
    xi = np.random.default_rng(1).integers(-100, 101, shape).astype(np.int32)
    np.testing.assert_array_equal(cp.cumsum(cp.array(xi), axis=1).get(), O.cumsum(xi, axis=1))


def test_cols_axis0_and_3d(cp):
    xi = np.random.default_rng(2).integers(-100, 101, (300, 70)).astype(np.int32)
    np.testing.assert_array_equal(cp.cumsum(cp.array(xi), axis=0).get(), O.cumsum(xi, axis=0))
    x3 = np.random.default_rng(3).integers(-9, 10, (4, 5, 6)).astype(np.int64)
    for ax in (0, 1, 2, None):
        np.testing.assert_array_equal(cp.cumsum(cp.array(x3), axis=ax).get(), O.cumsum(x3, axis=ax))


def test_dtypes(cp):
    for dt in (np.int16, np.uint16, np.uint32, np.bool_, np.int64):
        x = np.random.default_rng(4).integers(0, 3, 10000).astype(dt)
        got = cp.cumsum(cp.array(x))
        want = np.cumsum(x)
        assert got.dtype == want.dtype, dt
        np.testing.assert_array_equal(got.get(), want)
    # 5000: rows not a multiple of 16 elements (unaligned tile kernel);
    # 12400: 16-byte aligned, ragged last tile (pipelined tile kernel)
    for n in (5000, 12400):
        x = np.random.default_rng(5).uniform(0.999, 1.001, n).astype(np.float32)
        got = cp.cumprod(cp.array(x)).get()
        ref = np.cumprod(x.astype(np.float64))
        assert np.max(np.abs(got - ref) / ref) <= 1e-4
    x = np.random.default_rng(6).standard_normal(3 * 4096 + 48)
    got = cp.cumsum(cp.array(x)).get()
    assert got.dtype == np.float64
    ref = np.cumsum(x)
    assert np.max(np.abs(got - ref)) <= 1e-9 * np.abs(x).sum()


def test_repeated_calls_reuse_state(cp):
    x = np.random.default_rng(6).integers(-5, 6, 100000).astype(np.int32)
    X = cp.array(x)
    want = np.cumsum(x)
    for _ in range(5):
        np.testing.assert_array_equal(cp.cumsum(X).get(), want)
    cp.synchronize()


# Rows of at least 16 tiles in scans of at least 2^24 elements take the
# reduce-then-scan path (tile aggregates, a scan of the aggregates, tile
# scans with known carries).  Full-range int32 keeps the int64 carries exact;
# odd k takes the unaligned (scalar) tile path; a ragged last tile per row.
@pytest.mark.parametrize("rows,k", [(1, 1 << 25), (2, (1 << 23) + 2 * 4096 + 48), (3, (1 << 23) + 1000),
                                    (1, (1 << 24) + 5)])
def test_long_rows_reduce_then_scan(cp, rows, k):
    rng = np.random.default_rng(k + rows)
    x = rng.integers(-(1 << 31), (1 << 31) - 1, (rows, k), dtype=np.int64).astype(np.int32)
    X = cp.array(x)
    got = cp.cumsum(X, axis=1) if rows > 1 else cp.cumsum(X.reshape(-1)).reshape(rows, k)
    assert got.dtype == np.int64
    np.testing.assert_array_equal(got.get(), O.cumsum(x, axis=1))
    # values of both signs: the prefix crosses zero, so the bar's floor is
    # eps * sum|x| over the row (float32 eps), as stated for scans
    xf = rng.standard_normal((rows, k)).astype(np.float32)
    gf = cp.cumsum(cp.array(xf), axis=1).get()
    assert gf.dtype == np.float32
    ref = O.cumsum_f64(xf, axis=1)
    floor = np.finfo(np.float32).eps * np.abs(xf.astype(np.float64)).sum(axis=1, keepdims=True)
    assert np.max(np.abs(gf - ref) / np.maximum(np.abs(ref), floor)) <= 1e-4


def test_long_rows_carry_prod_and_dtypes(cp):
    from macmetalpy_b200 import reductions

    n = 1 << 25
    rng = np.random.default_rng(77)
    x = rng.integers(-1000, 1001, n).astype(np.int32)
    carry = 123456789012
    c = cp.array(np.array([carry], np.int64))
    got = reductions._scan(cp.array(x), 0, None, carry_ptr=c._ptr).get()
    np.testing.assert_array_equal(got, carry + np.cumsum(x, dtype=np.int64))
    xf = rng.uniform(0, 1, n).astype(np.float32)
    cf = cp.array(np.array([1.0e6], np.float64))
    gf = reductions._scan(cp.array(xf), 0, None, carry_ptr=cf._ptr).get()
    ref = 1.0e6 + np.cumsum(xf.astype(np.float64))
    assert np.max(np.abs(gf - ref) / ref) <= 1e-6
    # cumprod: signs only (exact), and values near 1
    s = rng.choice(np.array([-1, 1], np.int32), 1 << 24)
    np.testing.assert_array_equal(cp.cumprod(cp.array(s)).get(), np.cumprod(s.astype(np.int64)))
    p = rng.uniform(0.99999, 1.00001, 1 << 24).astype(np.float32)
    pref = np.cumprod(p.astype(np.float64))
    assert np.max(np.abs(cp.cumprod(cp.array(p)).get() - pref) / pref) <= 1e-4
    # other element types on the same path
    for dt in (np.int16, np.uint16, np.uint32, np.bool_, np.int64, np.float64):
        xd = rng.integers(0, 3, 1 << 24).astype(dt)
        gd = cp.cumsum(cp.array(xd))
        want = np.cumsum(xd)
        assert gd.dtype == want.dtype, dt
        np.testing.assert_array_equal(gd.get(), want)
    h = rng.uniform(0, 2e-3, 1 << 24).astype(np.float16)
    gh = cp.cumsum(cp.array(h)).get()
    assert gh.dtype == np.float16
    href = np.cumsum(h.astype(np.float64))
    assert np.max(np.abs(gh.astype(np.float64) - href) / np.maximum(href, 1e-3)) <= 2e-3


# Many rows under the stated scan bar: rows of one tile, ragged last tiles,
# rows of a few tiles and of hundreds; full-range int32 keeps the carries
# exact in int64.
@pytest.mark.parametrize("rows,k", [(300, 65536), (1000, 8192 + 16), (5000, 4096), (700, 3 * 4096 + 16),
                                    (3, (1 << 21) + 32)])
def test_many_rows(cp, rows, k):
    rng = np.random.default_rng(rows * 7 + k)
    x = rng.integers(-(1 << 31), (1 << 31) - 1, (rows, k), dtype=np.int64).astype(np.int32)
    got = cp.cumsum(cp.array(x), axis=1)
    np.testing.assert_array_equal(got.get(), O.cumsum(x, axis=1))
    xf = rng.standard_normal((rows, k)).astype(np.float32)
    gf = cp.cumsum(cp.array(xf), axis=1).get()
    ref = O.cumsum_f64(xf, axis=1)
    floor = np.finfo(np.float32).eps * np.abs(xf.astype(np.float64)).sum(axis=1, keepdims=True)
    assert np.max(np.abs(gf - ref) / np.maximum(np.abs(ref), floor)) <= 1e-4


# Signed data under the stated scan bar, |y - ref| / max(|ref|, eps * sum|x|)
# <= 1e-4 (eps: float32), at sizes the look-back kernel runs.  Float sums are
# f64 from the first element on; with f32 sums over each thread's 16
# elements these shapes gave 2.4e-4 to 8.7e-3.
@pytest.mark.parametrize("shape", [(1, 1 << 20), (64, 65536), (1, 1 << 22), (3, 40000)])
def test_signed_float_scan_bar(cp, shape):
    xf = np.random.default_rng(shape[1] + shape[0]).standard_normal(shape).astype(np.float32)
    gf = cp.cumsum(cp.array(xf), axis=1).get()
    ref = O.cumsum_f64(xf, axis=1)
    floor = np.finfo(np.float32).eps * np.abs(xf.astype(np.float64)).sum(axis=1, keepdims=True)
    assert np.max(np.abs(gf - ref) / np.maximum(np.abs(ref), floor)) <= 1e-4
    h = xf.astype(np.float16)
    gh = cp.cumsum(cp.array(h), axis=1).get().astype(np.float64)
    href = np.cumsum(h.astype(np.float64), axis=1)
    hfloor = np.finfo(np.float16).eps * np.abs(h.astype(np.float64)).sum(axis=1, keepdims=True)
    assert np.max(np.abs(gh - href) / np.maximum(np.abs(href), hfloor)) <= 1e-3


# One long aligned row ending in a partial tile: full-range int32 (int64
# carries exact), signed float32 under the scan bar, a carry-in, and cumprod.
def test_one_row_chunked_ragged(cp):
    from macmetalpy_b200 import reductions

    n = (1 << 24) + 37 * 4096 + 48
    rng = np.random.default_rng(91)
    x = rng.integers(-(1 << 31), (1 << 31) - 1, n, dtype=np.int64).astype(np.int32)
    np.testing.assert_array_equal(cp.cumsum(cp.array(x)).get(), O.cumsum(x))
    c = cp.array(np.array([-987654321], np.int64))
    got = reductions._scan(cp.array(x), 0, None, carry_ptr=c._ptr).get()
    np.testing.assert_array_equal(got, -987654321 + np.cumsum(x, dtype=np.int64))
    xf = rng.standard_normal(n).astype(np.float32)
    gf = cp.cumsum(cp.array(xf)).get()
    ref = O.cumsum_f64(xf)
    floor = np.finfo(np.float32).eps * np.abs(xf.astype(np.float64)).sum()
    assert np.max(np.abs(gf - ref) / np.maximum(np.abs(ref), floor)) <= 1e-4
    s = rng.choice(np.array([-1, 1], np.int32), n)
    np.testing.assert_array_equal(cp.cumprod(cp.array(s)).get(), np.cumprod(s.astype(np.int64)))


# Long rows on the reduce-then-scan path: one long row ending in a partial
# tile with a carry-in, many rows of exactly 16 tiles plus a ragged tail, and
# a few rows of 2^22 + 4096 elements.
@pytest.mark.parametrize("rows,k", [(1, (1 << 24) + 3 * 4096 + 32), (40, 16 * 4096 + 16), (5, (1 << 22) + 4096)])
def test_long_rows_ragged_and_carry(cp, rows, k):
    from macmetalpy_b200 import reductions

    rng = np.random.default_rng(rows + k)
    x = rng.integers(-(1 << 31), (1 << 31) - 1, (rows, k), dtype=np.int64).astype(np.int32)
    got = cp.cumsum(cp.array(x), axis=1)
    np.testing.assert_array_equal(got.get(), O.cumsum(x, axis=1))
    xf = rng.standard_normal((rows, k)).astype(np.float32)
    gf = cp.cumsum(cp.array(xf), axis=1).get()
    ref = O.cumsum_f64(xf, axis=1)
    floor = np.finfo(np.float32).eps * np.abs(xf.astype(np.float64)).sum(axis=1, keepdims=True)
    assert np.max(np.abs(gf - ref) / np.maximum(np.abs(ref), floor)) <= 1e-4
    if rows == 1:
        c = cp.array(np.array([555], np.int64))
        g1 = reductions._scan(cp.array(x.reshape(-1)), 0, None, carry_ptr=c._ptr).get()
        np.testing.assert_array_equal(g1, 555 + np.cumsum(x.reshape(-1), dtype=np.int64))


def test_long_scans_back_to_back(cp):
    """Consecutive long scans of different lengths and types on one stream,
    read back only at the end: the per-launch aggregate buffers and the
    look-back state of the aggregate scans do not leak between launches."""
    rng = np.random.default_rng(5)
    outs = []
    for n in ((1 << 24), (1 << 24) + 4096 * 37 + 16, (1 << 25) - 16, (1 << 24)):
        x = rng.integers(-50, 51, n).astype(np.int32)
        outs.append((cp.cumsum(cp.array(x)), x))
        xf = rng.uniform(-1, 1, n).astype(np.float32)
        outs.append((cp.cumsum(cp.array(xf)), xf))
    for got, x in outs:
        if x.dtype == np.int32:
            np.testing.assert_array_equal(got.get(), np.cumsum(x, dtype=np.int64))
        else:
            ref = O.cumsum_f64(x)
            floor = np.finfo(np.float32).eps * np.abs(x.astype(np.float64)).sum()
            assert np.max(np.abs(got.get() - ref) / np.maximum(np.abs(ref), floor)) <= 1e-4
    import ctypes

    from macmetalpy_b200 import _cuda_backend as cb

    code = ctypes.c_int(-1)
    assert cb.lib.mmp_check_device_error(ctypes.byref(code)) == 0 and code.value == 0
