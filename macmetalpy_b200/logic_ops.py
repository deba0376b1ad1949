"""Logic, predicate and comparison helpers (mirrors
``src/macmetalpy/logic_ops.py:32-66`` and ``math_ops.py:558-720``,
``ufunc_ops.py:352-354``).

Every function is a lazy fused node; the reductions among them
(``allclose``, ``array_equal``, ``count_nonzero``) fuse the predicate into
the one-launch reduction.  Semantics are the reference's CPU path (numpy):

* ``logical_and/or/xor/not``: numpy's bool results (``logic_ops.py:45-66``);
* ``isnan/isinf/isfinite/signbit``: bool (``math_ops.py:558-577``,
  ``ufunc_ops.py:352``);
* ``isclose``: numpy's ``|a - b| <= atol + rtol * |b|`` with the finite-b
  and exact-equality terms, ``equal_nan`` adding NaN pairs
  (``math_ops.py:639-660``);
* ``allclose`` / ``array_equal``: Python bool (``math_ops.py:663-690``);
* ``count_nonzero``: Python int, or an int64 (intp) array with ``axis``
  (``math_ops.py:693-720``);
* ``nan_to_num``: numpy's replacement values, default posinf/neginf the
  dtype's finite extremes (``math_ops.py:580-636``).
"""

from __future__ import annotations

import numpy as np

from .math_ops import _b, _u
from .ndarray import ndarray

__all__ = [
    "logical_and", "logical_or", "logical_xor", "logical_not", "isnan", "isinf", "isfinite",
    "signbit", "isclose", "allclose", "array_equal", "count_nonzero", "nan_to_num",
]

logical_and = _b("logical_and_op")
logical_or = _b("logical_or_op")
logical_xor = _b("logical_xor_op")
logical_not = _u("logical_not_op")
isnan = _u("isnan_op")
isinf = _u("isinf_op")
isfinite = _u("isfinite_op")
signbit = _u("signbit_op")


def _arr(x):
    from . import creation

    return x if isinstance(x, ndarray) else creation.asarray(np.asarray(x))


def isclose(a, b, rtol=1e-5, atol=1e-8, equal_nan=False):
    """numpy's isclose: b is first cast to ``result_type(b, 1.0)``; the
    tolerances are weak Python floats, so the test runs in the arrays'
    float type."""
    a, b = _arr(a), _arr(b)
    fdt = np.result_type(b.dtype, 1.0)
    if b.dtype != fdt:
        b = b.astype(fdt)
    rtol, atol = float(rtol), float(atol)
    r = logical_or(logical_and((abs(a - b) <= (atol + rtol * abs(b))), isfinite(b)), a == b)
    if equal_nan:
        r = logical_or(r, logical_and(isnan(a), isnan(b)))
    return r


def allclose(a, b, rtol=1e-5, atol=1e-8, equal_nan=False) -> bool:
    from . import reductions

    return bool(reductions.all(isclose(a, b, rtol=rtol, atol=atol, equal_nan=equal_nan)).get())


def array_equal(a, b, equal_nan=False) -> bool:
    from . import reductions

    a, b = _arr(a), _arr(b)
    if a.shape != b.shape:
        return False
    eq = a == b
    if equal_nan:
        eq = logical_or(eq, logical_and(isnan(a), isnan(b)))
    return bool(reductions.all(eq).get())


def count_nonzero(a, axis=None, keepdims=False):
    from . import reductions

    a = _arr(a)
    nz = a != 0 if a.dtype != np.bool_ else a
    r = reductions.sum(nz, axis=axis, keepdims=keepdims)
    if axis is None and not keepdims:
        return int(r.get())
    return r


def nan_to_num(x, copy=True, nan=0.0, posinf=None, neginf=None):
    x = _arr(x)
    if x.dtype.kind != "f":
        return x.copy() if copy else x
    fi = np.finfo(x.dtype)
    pos = fi.max if posinf is None else posinf
    neg = fi.min if neginf is None else neginf
    v = np.asarray([nan, pos, neg]).astype(x.dtype)
    r = ndarray._select(isnan(x), v[0], ndarray._select(x == np.inf, v[1],
                                                         ndarray._select(x == -np.inf, v[2], x)))
    if not copy:
        x[...] = r
        return x
    return r
