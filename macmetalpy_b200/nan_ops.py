"""NaN-aware reductions (mirrors ``src/macmetalpy/nan_ops.py:112-612``).

``nansum`` and ``nanmean`` are single masked reductions: NaN is skipped and
(for ``nanmean``) the non-NaN count is carried in the same pass.  The
reference runs ``nan_reduce_sum`` and finishes the partials on the CPU
(``nan_ops.py:89-98``), and builds ``nanmean`` from two replace kernels, two
sums, a divide, a compare and a ``where`` (``nan_ops.py:414-431``).
Integer inputs cannot hold NaN and use the plain reduction, as the
reference does (``nan_ops.py:132-134``).

The others follow numpy's nan-functions (the reference's CPU branch):
``nanprod``/``nancumsum``/``nancumprod`` replace NaN by the identity in a
fused select that feeds the reduction or scan (``nan_ops.py:171-270``);
``nanvar``/``nanstd`` give numpy's values -- the sum of squared deviations
of the non-NaN elements from their mean over ``count - ddof``, NaN where
that is <= 0 (``nan_ops.py:444-559``) -- in one pass that merges (count,
mean, M2) pairwise; ``nanargmax``/``nanargmin``
raise numpy's ``ValueError`` on an all-NaN slice, otherwise take the
arg-extreme with NaN replaced by -inf / +inf, returning a Python int without
an axis and numpy's int64 with one (``nan_ops.py:562-612``).
"""

from __future__ import annotations

import numpy as np

from .reductions import _asarray, _reduce

__all__ = ["nansum", "nanmean", "nanmax", "nanmin", "nanprod", "nancumsum", "nancumprod", "nanvar",
           "nanstd", "nanargmax", "nanargmin"]


def _out(r, out):
    if out is not None:
        out[...] = r
        return out
    return r


def _nan_as(a, v):
    """Lazy ``where(isnan(a), v, a)``."""
    from .logic_ops import isnan
    from .ndarray import ndarray

    return ndarray._select(isnan(a), v, a)


def nansum(a, axis=None, dtype=None, out=None, keepdims=False, initial=None, where=None):
    """Sum treating NaN as zero."""
    r = _reduce(a, "nansum", axis, keepdims, dtype=dtype)
    if initial is not None:
        r = r + initial
    if out is not None:
        out[...] = r
        return out
    return r


def nanmean(a, axis=None, dtype=None, out=None, keepdims=False, where=None):
    """Mean of the non-NaN elements (NaN where there are none)."""
    return _reduce(a, "nanmean", axis, keepdims, dtype=dtype, out=out)


def nanmax(a, axis=None, out=None, keepdims=False, initial=None, where=None):
    """Maximum ignoring NaN (NaN if all are NaN)."""
    return _reduce(a, "nanmax", axis, keepdims, out=out)


def nanmin(a, axis=None, out=None, keepdims=False, initial=None, where=None):
    """Minimum ignoring NaN (NaN if all are NaN)."""
    return _reduce(a, "nanmin", axis, keepdims, out=out)


def nanprod(a, axis=None, dtype=None, out=None, keepdims=False, initial=None, where=None):
    """Product treating NaN as one."""
    from . import reductions

    a = _asarray(a)
    if a.dtype.kind != "f":
        return reductions.prod(a, axis=axis, dtype=dtype, out=out, keepdims=keepdims)
    r = reductions.prod(_nan_as(a, 1), axis=axis, dtype=dtype, keepdims=keepdims)
    if initial is not None:
        r = r * initial
    return _out(r, out)


def nancumsum(a, axis=None, dtype=None, out=None):
    """Cumulative sum treating NaN as zero."""
    from . import reductions

    a = _asarray(a)
    if a.dtype.kind != "f":
        return reductions.cumsum(a, axis=axis, dtype=dtype, out=out)
    return reductions.cumsum(_nan_as(a, 0), axis=axis, dtype=dtype, out=out)


def nancumprod(a, axis=None, dtype=None, out=None):
    """Cumulative product treating NaN as one."""
    from . import reductions

    a = _asarray(a)
    if a.dtype.kind != "f":
        return reductions.cumprod(a, axis=axis, dtype=dtype, out=out)
    return reductions.cumprod(_nan_as(a, 1), axis=axis, dtype=dtype, out=out)


def nanvar(a, axis=None, dtype=None, out=None, ddof=0, keepdims=False, where=None, *, correction=None,
           mean=None):
    """Variance of the non-NaN elements: one pass (count, mean and M2 merged
    pairwise; NaN where fewer than ddof + 1 values remain).  The reference
    runs numpy's two-pass algorithm on the GPU (nan_ops.py:484-530)."""
    from . import reductions

    if correction is not None:
        ddof = correction
    a = _asarray(a)
    if a.dtype.kind != "f":
        return reductions.var(a, axis=axis, dtype=dtype, out=out, ddof=ddof, keepdims=keepdims)
    return _reduce(a, "nanvar", axis, keepdims, ddof=float(ddof), dtype=dtype, out=out)


def nanstd(a, axis=None, dtype=None, out=None, ddof=0, keepdims=False, where=None, *, correction=None,
           mean=None):
    """Standard deviation of the non-NaN elements (nan_ops.py:444-481)."""
    from . import reductions

    if correction is not None:
        ddof = correction
    a = _asarray(a)
    if a.dtype.kind != "f":
        return reductions.std(a, axis=axis, dtype=dtype, out=out, ddof=ddof, keepdims=keepdims)
    return _reduce(a, "nanstd", axis, keepdims, ddof=float(ddof), dtype=dtype, out=out)


def _nanarg(a, kind, fill, axis, out, keepdims):
    from . import reductions
    from .logic_ops import isnan

    a = _asarray(a)
    if a.dtype.kind != "f":
        return getattr(reductions, kind)(a, axis=axis, out=out, keepdims=keepdims)
    if a.size and bool(reductions.any(reductions.all(isnan(a), axis=axis)).get()):
        raise ValueError("All-NaN slice encountered")
    r = getattr(reductions, kind)(_nan_as(a, fill), axis=axis, keepdims=keepdims)
    if axis is None and not keepdims:
        return r
    return _out(r.astype(np.int64), out)


def nanargmax(a, axis=None, out=None, keepdims=False):
    """Index of the maximum ignoring NaN (first occurrence)."""
    return _nanarg(a, "argmax", -np.inf, axis, out, keepdims)


def nanargmin(a, axis=None, out=None, keepdims=False):
    """Index of the minimum ignoring NaN (first occurrence)."""
    return _nanarg(a, "argmin", np.inf, axis, out, keepdims)
