"""NaN-aware reductions (mirrors ``src/macmetalpy/nan_ops.py:112-168,379-432``).

``nansum`` and ``nanmean`` are single masked reductions: NaN is skipped and
(for ``nanmean``) the non-NaN count is carried in the same pass.  The
reference runs ``nan_reduce_sum`` and finishes the partials on the CPU
(``nan_ops.py:89-98``), and builds ``nanmean`` from two replace kernels, two
sums, a divide, a compare and a ``where`` (``nan_ops.py:414-431``).
Integer inputs cannot hold NaN and use the plain reduction, as the
reference does (``nan_ops.py:132-134``).
"""

from __future__ import annotations

from .reductions import _reduce

__all__ = ["nansum", "nanmean", "nanmax", "nanmin"]


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
