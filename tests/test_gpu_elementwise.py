"""Fused elementwise kernels vs the oracle: size sweeps across vector and
block boundaries, broadcasting, strided/negative-stride views, scalars,
dtype promotion, casts, in-place ops and the fusion depth cap."""

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 3, 4, 5, 31, 32, 33, 255, 256, 257, 1023, 1024, 1025, 4097, 65537, (1 << 20) + 3]


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    return cp


def _ab(n, dtype, seed=0):
    rng = np.random.default_rng(seed)
    if np.dtype(dtype).kind == "f":
        a = rng.uniform(-1000, 1000, n).astype(dtype)
        b = (rng.uniform(1, 50, n) * rng.choice([-1, 1], n)).astype(dtype)
    else:
        a = rng.integers(-1000, 1000, n).astype(dtype)
        b = (rng.integers(1, 50, n) * rng.choice([-1, 1], n)).astype(dtype)
    return a, b


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("dtype", [np.float32, np.int32])
def test_binary_sweep_bit_exact(cp, n, dtype):
    a, b = _ab(n, dtype, seed=n)
    A, B = cp.array(a), cp.array(b)
    np.testing.assert_array_equal(cp.add(A, B).get(), O.add(a, b))
    np.testing.assert_array_equal(cp.floor_divide(A, B).get(), O.floor_divide(a, b))
    np.testing.assert_array_equal((A % B).get(), O.mod(a, b))
    if dtype == np.float32:
        got = cp.logaddexp(A, B).get()
        ref64 = np.logaddexp(a.astype(np.float64), b.astype(np.float64))
        # <= 2 ulp except where the result cancels towards 0 (x ~ -log1p(e^-|d|)),
        # where the float32 algorithm itself (numpy's, the reference's) loses digits:
        # there the bar is 2 ulp of the larger operand
        scale = np.maximum(np.abs(ref64), np.maximum(np.abs(a), np.abs(b)).astype(np.float64))
        err = np.abs(got.astype(np.float64) - ref64) / np.spacing(scale.astype(np.float32)).astype(np.float64)
        assert err.max(initial=0) <= 2
        refnp = O.logaddexp(a, b).astype(np.float64)
        assert (np.abs(got.astype(np.float64) - refnp) <= 2 * np.spacing(scale.astype(np.float32))).all()


@pytest.mark.parametrize("dtype", [np.int16, np.uint16, np.int64, np.uint32, np.float16, np.float64])
def test_other_dtypes(cp, dtype):
    rng = np.random.default_rng(7)
    a = (rng.integers(1, 100, 3000)).astype(dtype)
    b = (rng.integers(1, 9, 3000)).astype(dtype)
    A, B = cp.array(a), cp.array(b)
    for op in ("add", "subtract", "multiply", "floor_divide", "maximum", "minimum"):
        got = getattr(cp, op)(A, B).get()
        want = getattr(np, op)(a, b)
        assert got.dtype == want.dtype, op
        np.testing.assert_array_equal(got, want, err_msg=op)
    np.testing.assert_array_equal((A % B).get(), O.mod(a, b))


@pytest.mark.parametrize("op", ["sqrt", "exp", "log", "sin", "cos", "tanh", "arctan", "log1p", "expm1", "cbrt",
                                "exp2", "log2", "log10", "sinh", "cosh", "arcsinh"])
def test_unary_transcendental_ulp(cp, op):
    rng = np.random.default_rng(3)
    x = rng.uniform(0.01, 5, 50000).astype(np.float32)
    got = getattr(cp, op)(cp.array(x)).get()
    ref = getattr(np, op)(x.astype(np.float64))
    assert O.ulp_error(got, ref).max() <= 2.0, op


@pytest.mark.parametrize("op", ["floor", "ceil", "trunc", "rint", "abs", "negative", "square", "sign",
                                "reciprocal", "degrees", "radians"])
def test_unary_exact(cp, op):
    rng = np.random.default_rng(4)
    x = (rng.standard_normal(10000) * 50).astype(np.float32)
    x[:6] = [0.0, -0.0, 0.5, -0.5, 1.5, 2.5]
    got = getattr(cp, op)(cp.array(x)).get()
    want = getattr(np, op)(x)
    np.testing.assert_array_equal(got, want)


def test_maximum_minimum_nan_rules(cp):
    a = np.array([1, np.nan, 3, -0.0, 0.0, np.nan], np.float32)
    b = np.array([np.nan, 2, 1, 0.0, -0.0, np.nan], np.float32)
    A, B = cp.array(a), cp.array(b)
    for op in ("maximum", "minimum", "fmax", "fmin"):
        got = getattr(cp, op)(A, B).get()
        want = getattr(np, op)(a, b)
        np.testing.assert_array_equal(got, want, err_msg=op)


@pytest.mark.parametrize("shape_a,shape_b", [((257, 1), (1, 1000)), ((2, 3), (3,)), ((2, 1, 3), (3, 1)),
                                             ((1,), (2, 3)), ((5, 1, 7, 1), (1, 6, 1, 9)), ((), (4, 4))])
def test_broadcast(cp, shape_a, shape_b):
    rng = np.random.default_rng(5)
    a = rng.standard_normal(shape_a).astype(np.float32)
    b = rng.standard_normal(shape_b).astype(np.float32)
    np.testing.assert_array_equal((cp.array(a) + cp.array(b)).get(), a + b)
    np.testing.assert_array_equal((cp.array(a) * cp.array(b) - 1.5).get(), a * b - np.float32(1.5))


def test_strided_views(cp):
    rng = np.random.default_rng(6)
    a = rng.standard_normal((64, 96)).astype(np.float32)
    A = cp.array(a)
    for view, nview in ((A.T, a.T), (A[::2, 1::3], a[::2, 1::3]), (A[::-1], a[::-1]), (A[:, ::-2], a[:, ::-2]),
                        (A[5], a[5]), (A[:, 7], a[:, 7]), (A[None, 3:9, :, None], a[None, 3:9, :, None])):
        np.testing.assert_array_equal(cp.exp(view).get(), np.exp(nview).astype(np.float32)
                                      if False else cp.exp(cp.array(nview.copy())).get())
        np.testing.assert_array_equal((view + 1).get(), nview + np.float32(1))
        np.testing.assert_array_equal(view.get(), nview)


def test_scalars_and_promotion(cp):
    a = np.arange(1, 101, dtype=np.int32)
    A = cp.array(a)
    assert (A + 1).dtype == np.int32
    assert (A * 2.5).dtype == np.float64  # numpy: int32 * python float -> float64
    np.testing.assert_array_equal((A * 2.5).get(), a * 2.5)
    assert (A / A).dtype == np.float64
    f = cp.array(a.astype(np.float32))
    assert (f + 1).dtype == np.float32
    assert (f * np.float64(2)).dtype == np.float64
    np.testing.assert_array_equal((f ** 2).get(), a.astype(np.float32) ** 2)
    np.testing.assert_array_equal((2 - f).get(), 2 - a.astype(np.float32))


def test_downcast_config(cp):
    cp.set_config(float64_behavior="downcast", warn_on_downcast=False)
    A = cp.array(np.arange(10, dtype=np.int32))
    assert (A * 2.5).dtype == np.float32
    assert cp.array(np.ones(3)).dtype == np.float32


def test_astype_and_cast_fusion(cp):
    x = np.linspace(-3, 3, 1001).astype(np.float32)
    X = cp.array(x)
    np.testing.assert_array_equal(X.astype(np.int32).get(), x.astype(np.int32))
    np.testing.assert_array_equal(X.astype(np.float16).get(), x.astype(np.float16))
    np.testing.assert_array_equal((X > 0).get(), x > 0)
    np.testing.assert_array_equal(cp.where(X > 0, X, 0).get(), np.where(x > 0, x, 0))


def test_inplace_and_setitem(cp):
    a = np.arange(24, dtype=np.float32).reshape(4, 6)
    A = cp.array(a)
    A += 1
    a += 1
    np.testing.assert_array_equal(A.get(), a)
    A[1] = 7
    a[1] = 7
    A[:, ::2] = cp.array(np.full((4, 3), -1, np.float32))
    a[:, ::2] = -1
    np.testing.assert_array_equal(A.get(), a)


def test_fusion_depth_cap(cp):
    x = np.random.default_rng(8).standard_normal(1000).astype(np.float32) * 0.1
    X = cp.array(x)
    r, rn = X, x
    for _ in range(40):  # deeper than _MAX_DEPTH = 16
        r = r + 0.01
        rn = rn + np.float32(0.01)
    np.testing.assert_array_equal(r.get(), rn)


def test_shared_subexpression(cp):
    x = np.random.default_rng(9).standard_normal(5000).astype(np.float32)
    X = cp.array(x)
    s = cp.sin(X)
    r = s * s + s
    sn = np.sin(x.astype(np.float64))
    # absolute bar: the sum cancels near s = -1 and s = 0
    assert np.max(np.abs(r.get() - (sn * sn + sn))) <= 4 * np.spacing(np.float32(2))


def test_floor_divide_mod_magnitude_sweep(cp):
    """Bit-exact float32 floor_divide / mod across quotient magnitudes (both
    sides of the 2^20 fast-path bound), tiny and huge divisors, subnormals,
    signed zeros, infinities and NaN."""
    rng = np.random.default_rng(11)
    n = 1 << 18
    ea = rng.uniform(-40, 40, n)
    eb = rng.uniform(-40, 40, n)
    a = (rng.choice([-1, 1], n) * rng.uniform(1, 2, n) * 2.0 ** ea).astype(np.float32)
    b = (rng.choice([-1, 1], n) * rng.uniform(1, 2, n) * 2.0 ** eb).astype(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 3.4e38, 1.0, -1.0, 2 ** 20, 2 ** 21],
                       np.float32)
    a[:144] = np.repeat(special, 12)
    b[:144] = np.tile(special, 12)
    A, B = cp.array(a), cp.array(b)
    np.testing.assert_array_equal(cp.floor_divide(A, B).get(), O.floor_divide(a, b))
    np.testing.assert_array_equal((A % B).get(), O.mod(a, b))
    ai = rng.integers(-2 ** 31, 2 ** 31, n).astype(np.int32)
    bi = rng.integers(-2 ** 31, 2 ** 31, n).astype(np.int32)
    bi[:100] = rng.integers(-3, 4, 100)
    ai[:8] = [-2 ** 31, -2 ** 31, 2 ** 31 - 1, 0, 7, -7, 5, -5]
    bi[:8] = [-1, 1, -1, 0, 0, 0, -1, 1]
    Ai, Bi = cp.array(ai), cp.array(bi)
    np.testing.assert_array_equal(cp.floor_divide(Ai, Bi).get(), O.floor_divide(ai, bi))
    np.testing.assert_array_equal((Ai % Bi).get(), O.mod(ai, bi))


def test_int32_floor_divide_fast_path_boundaries(cp):
    """int32 floor_divide / % around the float fast path's bounds (|a| < 2^21,
    |b| < 2^24): bit-exact against numpy on both sides."""
    rng = np.random.default_rng(12)
    n = 1 << 20
    mags = np.array([1, 7, 1000, (1 << 21) - 1, 1 << 21, (1 << 24) - 1, 1 << 24, (1 << 31) - 1], np.int64)
    a = (rng.choice(mags, n) - rng.integers(0, 3, n)) * rng.choice([-1, 1], n)
    b = (rng.choice(mags, n) - rng.integers(0, 3, n)) * rng.choice([-1, 1], n)
    a = np.clip(a, -(1 << 31), (1 << 31) - 1).astype(np.int32)
    b = np.clip(b, -(1 << 31), (1 << 31) - 1).astype(np.int32)
    b[b == 0] = 3
    A, B = cp.array(a), cp.array(b)
    np.testing.assert_array_equal(cp.floor_divide(A, B).get(), O.floor_divide(a, b))
    np.testing.assert_array_equal((A % B).get(), O.mod(a, b))
    small = rng.integers(-(1 << 21) + 1, 1 << 21, n).astype(np.int32)
    sb = rng.integers(1, 1 << 24, n).astype(np.int32) * rng.choice(np.array([-1, 1], np.int32), n)
    np.testing.assert_array_equal(cp.floor_divide(cp.array(small), cp.array(sb)).get(), O.floor_divide(small, sb))
