"""The remaining NaN-aware reductions and scans on the device against the
reference's golden vectors (tests/golden/golden_nan_v1.npz) and against the
oracle on larger seeded inputs: nanprod, nancumsum, nancumprod, nanvar,
nanstd (1e-4 relative, the float reduction bar; NaN where numpy gives NaN),
nanargmax / nanargmin (exact, numpy's ValueError on an all-NaN slice)."""

import os
import warnings

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

N = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_nan_v1.npz"))
warnings.simplefilter("ignore", RuntimeWarning)


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    return cp


def close(got, want, rtol=1e-4):
    got = got.get() if hasattr(got, "get") else np.asarray(got)
    want = np.asarray(want)
    assert got.dtype == want.dtype, (got.dtype, want.dtype)
    assert got.shape == want.shape, (got.shape, want.shape)
    g, w = got.astype(np.float64), want.astype(np.float64)
    assert np.array_equal(np.isnan(g), np.isnan(w))
    ok = ~np.isnan(w)
    if ok.any():
        assert np.max(np.abs(g[ok] - w[ok]) / np.maximum(np.abs(w[ok]), 1e-6)) <= rtol


def scan_close(got, want, x, axis=-1, rtol=1e-4):
    """Scan bar: |y_i - ref_i| / max(|ref_i|, running sum of |x|) -- a prefix
    of signed values crosses zero, where an elementwise relative error is not
    defined by the data."""
    got = got.get()
    assert got.dtype == np.asarray(want).dtype
    scale = np.cumsum(np.abs(np.nan_to_num(np.asarray(x, np.float64))), axis=axis)
    g, w = got.astype(np.float64), np.asarray(want, np.float64)
    assert np.max(np.abs(g - w) / np.maximum(np.maximum(np.abs(w), scale), 1e-30)) <= rtol


def test_golden_nanprod_and_scans(cp):
    P, V, M, MI = (cp.array(N[k]) for k in ("p", "v", "m", "mi"))
    close(cp.nanprod(P), N["nanprod"])
    close(cp.nanprod(P, axis=0), N["nanprod_ax0"])
    close(cp.nanprod(P, axis=1), N["nanprod_ax1"])
    scan_close(cp.nancumsum(V), N["nancumsum"], N["v"])
    scan_close(cp.nancumsum(M, axis=1), N["nancumsum_ax1"], N["m"], axis=1)
    close(cp.nancumprod(P, axis=0), N["nancumprod_ax0"])
    np.testing.assert_array_equal(cp.nancumsum(MI).get(), N["nancumsum_i"])


def test_golden_nanvar_nanstd(cp):
    M, MI = cp.array(N["m"]), cp.array(N["mi"])
    for ddof in (0, 1):
        close(cp.nanvar(M, ddof=ddof), N[f"nanvar_d{ddof}"])
        close(cp.nanvar(M, axis=0, ddof=ddof), N[f"nanvar_ax0_d{ddof}"])
        close(cp.nanvar(M, axis=1, ddof=ddof), N[f"nanvar_ax1_d{ddof}"])
        close(cp.nanstd(M, axis=1, ddof=ddof), N[f"nanstd_ax1_d{ddof}"])
    close(cp.nanvar(MI), N["nanvar_i"])


def test_golden_nanarg(cp):
    V, MM, MI, M = (cp.array(N[k]) for k in ("v", "mm", "mi", "m"))
    r = cp.nanargmax(V)
    assert isinstance(r, int) and r == int(N["nanargmax"])
    assert cp.nanargmin(V) == int(N["nanargmin"])
    got = cp.nanargmax(MM, axis=1)
    assert got.dtype == np.int64
    np.testing.assert_array_equal(got.get(), N["nanargmax_ax1"])
    np.testing.assert_array_equal(cp.nanargmin(MM, axis=0).get(), N["nanargmin_ax0"])
    gi = cp.nanargmax(MI, axis=0)
    assert gi.dtype == np.int32
    np.testing.assert_array_equal(gi.get(), N["nanargmax_i_ax0"])
    with pytest.raises(ValueError):
        cp.nanargmax(M, axis=1)
    with pytest.raises(ValueError):
        cp.nanargmin(cp.array(np.full(10, np.nan, np.float32)))


@pytest.mark.parametrize("shape", [(1 << 20,), (1000, 3000), (4097, 5)])
def test_large_vs_oracle(cp, shape):
    rng = np.random.default_rng(sum(shape))
    x = rng.standard_normal(shape).astype(np.float32)
    x[rng.random(shape) < 0.02] = np.nan
    X = cp.array(x)
    axes = [None] + list(range(len(shape)))
    for ax in axes:
        close(cp.nanvar(X, axis=ax), O.nanvar(x, axis=ax))
        close(cp.nanstd(X, axis=ax, ddof=1), O.nanstd(x, axis=ax, ddof=1))
        ga, wa = cp.nanargmax(X, axis=ax), O.nanargmax(x, axis=ax)
        if ax is None:
            assert ga == wa
        else:
            np.testing.assert_array_equal(ga.get(), wa)
    y = np.abs(x[..., :64] if len(shape) > 1 else x[:4096]) * np.float32(0.01) + np.float32(0.995)
    close(cp.nanprod(cp.array(y), axis=-1), O.nanprod(y, axis=-1), rtol=1e-3)
    c = cp.nancumsum(X, axis=-1).get().astype(np.float64)
    ref = np.nancumsum(x.astype(np.float64), axis=-1)
    scale = np.nancumsum(np.abs(x.astype(np.float64)), axis=-1)
    assert np.max(np.abs(c - ref) / np.maximum(scale, 1e-6)) <= 1e-4


def test_nanvar_one_pass_edges(cp):
    """One-pass nanvar: the first element NaN with a large common offset
    (no shift to lean on), all-NaN rows and dof <= 0 give NaN, float16 and
    float64 inputs, and a fused expression as input."""
    rng = np.random.default_rng(21)
    x = (rng.standard_normal((64, 5000)) + 1.0e4).astype(np.float32)
    x[rng.random(x.shape) < 0.05] = np.nan
    x[:, 0] = np.nan
    x[7] = np.nan                      # an all-NaN row
    x[9, 1:] = np.nan                  # one value left: ddof=1 gives NaN
    X = cp.array(x)
    for ax in (None, 0, 1):
        for ddof in (0, 1):
            close(cp.nanvar(X, axis=ax, ddof=ddof), O.nanvar(x, axis=ax, ddof=ddof))
    close(cp.nanstd(X, axis=1), O.nanstd(x, axis=1))
    # float16: scale kept small so that numpy's own float16 sum of squares
    # does not overflow to inf (this library accumulates in f32/f64)
    for dt, sc in ((np.float16, 0.3), (np.float64, 3.0)):
        xd = (rng.standard_normal(30000) * sc).astype(dt)
        xd[::7] = np.nan
        close(cp.nanvar(cp.array(xd)), O.nanvar(xd), rtol=3e-3 if dt == np.float16 else 1e-6)
    y = rng.standard_normal(1 << 20).astype(np.float32)
    y[::13] = np.nan
    Y = cp.array(y)
    close(cp.nanvar(Y * 2 + 1), O.nanvar(y * np.float32(2) + np.float32(1)))
