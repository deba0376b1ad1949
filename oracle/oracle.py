"""CPU oracle for the macmetalpy_b200 hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs
(``cpu_baseline`` and ``--impl reference``) may import this module, and only
as the checker / the timed CPU baseline.  The product path
(``macmetalpy_b200``) never imports it and has no CPU fallback.

It restates, with numpy, what the reference computes on its CPU path for
each op of the hot path (the reference's Metal path cannot run on Linux; its
CPU branch is plain numpy dispatch, ``ndarray.py:960-1159``).  Each function
cites the reference code it follows.  Parity is pinned: ``tests/
test_oracle_golden.py`` checks every function against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference itself.

For float reductions and scans the target tolerance is stated against a
float64-accumulated result (the ``*_f64`` helpers), because the reference's
float32 CPU results drift at the BASELINE sizes (a sequential float32
``cumsum`` of 2^30 values in U(0,1) stalls once the prefix passes 2^24).
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "resolve_dtype", "c1_expression", "add", "floor_divide", "mod", "logaddexp", "broadcast_add",
    "reduce_sum", "reduce_mean", "reduce_var", "argmax", "argmax_axis", "nansum", "nanmean",
    "cumsum", "matmul", "sum_f64", "mean_f64", "var_f64", "cumsum_f64", "matmul_f64", "ulp_error",
]


def resolve_dtype(dtype, float64_behavior: str = "cpu_fallback", default_float: str = "float32"):
    """``_dtypes.resolve_dtype`` (src/macmetalpy/_dtypes.py:77-136)."""
    if dtype is None:
        return np.dtype(default_float)
    dt = np.dtype(dtype)
    if dt == np.float64:
        return np.dtype(default_float) if float64_behavior == "downcast" else dt
    if dt == np.int8:
        return np.dtype(np.int16)
    if dt == np.uint8:
        return np.dtype(np.uint16)
    return dt


# ---------------------------------------------------------------- elementwise


def c1_expression(x):
    """``sqrt(abs(x)) + exp(-x**2)`` as the reference evaluates it op by op
    (math_ops.sqrt/exp ``math_ops.py:15-34`` -> ``_unary_op`` CPU branch
    ``ndarray.py:1161-1180``; ``x**2`` -> ``__pow__`` ``ndarray.py:1371``)."""
    x = np.asarray(x)
    return np.sqrt(np.abs(x)) + np.exp(-(x * x))


def add(a, b):
    """``ufunc_ops.add`` (ufunc_ops.py:38-45) -> numpy add."""
    return np.add(a, b)


def floor_divide(a, b):
    """``ufunc_ops.floor_divide`` (ufunc_ops.py:101-108) -> numpy floor_divide
    (floor semantics; integer division by zero gives 0)."""
    with np.errstate(all="ignore"):
        return np.floor_divide(a, b)


def mod(a, b):
    """``math_ops.mod`` / ``ndarray.__mod__`` (math_ops.py:540-548,
    ndarray.py:2525-2530): ``x1 - floor_divide(x1, x2) * x2``, each step a
    numpy op in the array dtype (not ``np.remainder``)."""
    with np.errstate(all="ignore"):
        fd = np.floor_divide(a, b)
        return a - fd * b


def logaddexp(a, b):
    """``ufunc_ops.logaddexp`` (ufunc_ops.py:238-244) -> numpy logaddexp."""
    return np.logaddexp(a, b)


def broadcast_add(a, b):
    """``_binary_op`` with ``needs_broadcast`` (ndarray.py:1062-1065): numpy
    broadcasting add."""
    return np.add(a, b)


# ---------------------------------------------------------------- reductions


def reduce_sum(a, axis=None):
    """``reductions.sum`` CPU branch (reductions.py:86-100): ``np.sum`` --
    int32 accumulates and returns int64."""
    return np.sum(a, axis=axis)


def reduce_mean(a, axis=None):
    """``reductions.mean`` CPU branch (reductions.py:128-150): ``np.mean``."""
    return np.mean(a, axis=axis)


def reduce_var(a, axis=None, ddof=0):
    """``reductions.var`` CPU branch (reductions.py:540-556): ``np.var``."""
    return np.var(a, axis=axis, ddof=ddof)


def argmax(a):
    """``reductions.argmax(axis=None)`` (reductions.py:381-418): a Python
    int, first occurrence, the first NaN wins (numpy)."""
    return int(np.argmax(a))


def argmax_axis(a, axis):
    """``reductions.argmax(axis=k)`` -> ``_reduce_axis(..., out_dtype=int32)``
    (reductions.py:410, ndarray.py:2015-2035): numpy argmax cast to int32."""
    return np.asarray(np.argmax(a, axis=axis), dtype=np.int32)


def nansum(a, axis=None):
    """``nan_ops.nansum`` (nan_ops.py:112-168) -> ``np.nansum``."""
    return np.nansum(a, axis=axis)


def nanmean(a, axis=None):
    """``nan_ops.nanmean`` (nan_ops.py:379-432) -> ``np.nanmean`` (NaN when
    a slice holds no number)."""
    with np.errstate(all="ignore"):
        import warnings

        with warnings.catch_warnings():
            warnings.simplefilter("ignore", RuntimeWarning)
            return np.nanmean(a, axis=axis)


def cumsum(a, axis=None):
    """``reductions.cumsum`` CPU branch (reductions.py:661-681):
    ``np.cumsum`` (int32 -> int64)."""
    return np.cumsum(a, axis=axis)


def matmul(a, b):
    """``linalg_top.matmul`` CPU branch (linalg_top.py:94-111): ``np.matmul``
    (float16 in, float16 out)."""
    return np.matmul(a, b)


# ---------------------------------------------------------------- float64 references


def sum_f64(a, axis=None):
    return np.sum(np.asarray(a, dtype=np.float64), axis=axis)


def mean_f64(a, axis=None):
    return np.mean(np.asarray(a, dtype=np.float64), axis=axis)


def var_f64(a, axis=None, ddof=0):
    return np.var(np.asarray(a, dtype=np.float64), axis=axis, ddof=ddof)


def cumsum_f64(a, axis=None):
    return np.cumsum(np.asarray(a, dtype=np.float64), axis=axis)


def matmul_f64(a, b):
    return np.matmul(np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64))


def ulp_error(got, ref64) -> np.ndarray:
    """|got - ref| in units of the float32 ulp at the float32-rounded
    reference (the <= 2 ulp bar for transcendentals)."""
    got = np.asarray(got, dtype=np.float32)
    ref32 = np.asarray(ref64, dtype=np.float32)
    spacing = np.spacing(np.abs(ref32)).astype(np.float64)
    spacing[spacing == 0] = np.finfo(np.float32).tiny
    err = np.abs(got.astype(np.float64) - np.asarray(ref64, dtype=np.float64)) / spacing
    both_nan = np.isnan(got) & np.isnan(ref32)
    same_inf = np.isinf(got) & np.isinf(ref32) & (np.sign(got) == np.sign(ref32))
    err[both_nan | same_inf] = 0.0
    return err
