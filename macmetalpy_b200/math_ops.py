"""Math functions (mirrors ``src/macmetalpy/math_ops.py:15-103,540-548``).

Every function builds a lazy fused node (``ndarray._elementwise``).
``mod``/``remainder`` (and ``%``) compute the reference's own composite
``x1 - floor_divide(x1, x2) * x2`` (``math_ops.py:540-548``), each step
rounded to the dtype as the reference's three kernels round it, but as ONE
fused kernel (``csrc/mmp_fused_ops.cuh``); for floats this is not numpy's
``remainder``, and the golden vectors recorded from the reference pin it.
``dot`` of 1-D arrays is a fused multiply + sum reduction (the reference's
``_reduce_dot``, ``ndarray.py:1965-2013``); 2-D ``dot`` is ``matmul``.
"""

from __future__ import annotations

import numpy as np

from .ndarray import _elementwise_fast, ndarray

__all__ = [
    "sqrt", "exp", "log", "abs", "absolute", "fabs", "power", "negative", "positive", "sign", "square",
    "sin", "cos", "tan", "arcsin", "arccos", "arctan", "sinh", "cosh", "tanh", "log2", "log10",
    "floor", "ceil", "mod", "remainder", "dot", "where", "clip", "divmod", "around", "round", "round_",
]


def _u(op):
    def f(x, out=None, **kwargs):
        r = _elementwise_fast(op, (x,))
        if r is None:
            r = ndarray._elementwise(op, x)
        if out is not None:
            out[...] = r
            return out
        return r
    f.__name__ = op[:-3]
    f.__doc__ = f"Elementwise {op[:-3]} (lazy, fused)."
    return f


def _b(op):
    def f(x1, x2, out=None, **kwargs):
        r = ndarray._elementwise(op, x1, x2) if not (op == "pow_op" and isinstance(x1, ndarray)) \
            else x1._binary_op(x2, op)
        if out is not None:
            out[...] = r
            return out
        return r
    f.__name__ = op[:-3]
    f.__doc__ = f"Elementwise {op[:-3]} (lazy, fused)."
    return f


sqrt = _u("sqrt_op")
exp = _u("exp_op")
log = _u("log_op")
absolute = _u("abs_op")
abs = absolute
negative = _u("negative_op")
positive = _u("positive_op")
sign = _u("sign_op")
square = _u("square_op")
sin = _u("sin_op")
cos = _u("cos_op")
tan = _u("tan_op")
arcsin = _u("asin_op")
arccos = _u("acos_op")
arctan = _u("atan_op")
sinh = _u("sinh_op")
cosh = _u("cosh_op")
tanh = _u("tanh_op")
log2 = _u("log2_op")
log10 = _u("log10_op")
floor = _u("floor_op")
ceil = _u("ceil_op")
power = _b("pow_op")
mod = _b("mod_op")
remainder = mod


def fabs(x, out=None, **kwargs):
    r = ndarray._elementwise("abs_op", x)
    return r if r.dtype.kind == "f" else r.astype(np.float64)


def divmod(x1, x2):
    return ndarray._elementwise("floor_divide_op", x1, x2), ndarray._elementwise("mod_op", x1, x2)


def dot(a, b, out=None):
    """Dot product: fused multiply-sum for 1-D, matmul otherwise."""
    from . import creation, linalg_top, reductions
    a = creation.asarray(a)
    b = creation.asarray(b)
    if a.ndim == 0 or b.ndim == 0:
        r = a * b
    elif a.ndim == 1 and b.ndim == 1:
        if a.shape != b.shape:
            raise ValueError(f"shapes {a.shape} and {b.shape} not aligned")
        r = reductions.sum(a * b)
    else:
        r = linalg_top.matmul(a, b)
    if out is not None:
        out[...] = r
        return out
    return r


def where(condition, x=None, y=None):
    """``where(c, x, y)`` as a fused select: c*x + (1-c)*y is NOT used; the
    select is built from comparison masks so NaN/inf pass through."""
    if x is None and y is None:  # where(condition) is nonzero(condition)
        from . import _advindex
        from . import creation
        c = condition if isinstance(condition, ndarray) else creation.asarray(np.asarray(condition))
        return _advindex.nonzero(c)
    if x is None or y is None:
        raise ValueError("either both or neither of x and y should be given")
    from . import creation
    c = condition if isinstance(condition, ndarray) else creation.asarray(np.asarray(condition))
    cb = c if c.dtype == np.bool_ else (c != 0)
    return ndarray._select(cb, x, y)


def clip(a, a_min=None, a_max=None, out=None, **kwargs):
    from . import creation
    r = creation.asarray(a).clip(a_min, a_max)
    if out is not None:
        out[...] = r
        return out
    return r


def around(a, decimals=0, out=None):
    """Round to ``decimals`` places (math_ops.py, numpy's ``around``): for
    floats ``rint(a * 10**d) / 10**d`` (``a / 10**-d`` then ``* 10**-d`` for
    negative d), each step in the array's dtype as numpy evaluates it; for
    integers a copy when d >= 0, else the same steps in float64 and a cast
    back."""
    from .creation import asarray

    a = asarray(a)
    d = int(decimals)
    if a.dtype.kind in "iub":
        if d >= 0:
            r = a.copy()
        else:
            f = float(10 ** (-d))  # numpy rounds integers in float64, then casts back
            r = (ndarray._elementwise("rint_op", a.astype(np.float64) / f) * f).astype(a.dtype)
    elif d == 0:
        r = ndarray._elementwise("rint_op", a)
    elif d > 0:
        f = float(10 ** d)
        r = ndarray._elementwise("rint_op", a * f) / f
    else:
        f = float(10 ** (-d))
        r = ndarray._elementwise("rint_op", a / f) * f
    if out is not None:
        out[...] = r
        return out
    return r


round = around
round_ = around

