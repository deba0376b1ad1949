"""Sorting and searching (mirrors ``src/macmetalpy/sorting.py:22-272`` and
``ndarray.sort/argsort/searchsorted``, ``ndarray.py:2393-2412``).

``sort`` / ``argsort`` run the device radix sort (``mmp_sort``) for every
dtype, size and axis: the sorted axis is moved last (one fused copy when it
is not already), then every row is sorted in one call.  Results are numpy's
(the reference's CPU branch): NaN sorts last, ``argsort`` is stable and
int64 -- numpy's ``kind="stable"``; numpy's default kind orders ties
unspecified, the reference's GPU bitonic branch (``sorting.py:57-190``)
returns int32 and has no defined NaN order.  ``searchsorted`` is one binary
search per query in numpy's order (NaN last), both operands in their common
dtype, int64 result (``sorting.py:218-272``).
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _cuda_backend as _cb
from ._dtypes import MMP_CODES
from .ndarray import ndarray

__all__ = ["sort", "argsort", "searchsorted", "msort"]


def _asarray(a) -> ndarray:
    from .creation import asarray

    return a if isinstance(a, ndarray) else asarray(np.asarray(a))


def _rows_last(a: ndarray, axis):
    """(contiguous array with the sorted axis last, axis index, original
    ndim).  ``axis=None`` sorts the flattened array."""
    if axis is None:
        return a.reshape(-1)._ensure_contiguous(), 0, 1
    nd = a.ndim
    if nd == 0:
        raise np.exceptions.AxisError(axis, 0)
    ax = int(axis)
    if not -nd <= ax < nd:
        raise np.exceptions.AxisError(axis, nd)
    ax %= nd
    if ax != nd - 1:
        a = a.swapaxes(ax, nd - 1)
    return a._ensure_contiguous(), ax, nd


def _back(r: ndarray, ax: int, nd: int) -> ndarray:
    if ax != nd - 1:
        r = r.swapaxes(ax, nd - 1)._ensure_contiguous()
    return r


def _run(src: ndarray, values: bool) -> ndarray:
    cols = src._shape[-1] if src.ndim else 1
    rows = src.size // cols if cols else 0
    if values:
        res = ndarray._empty(src._shape, src._dtype)
        y, idx = ctypes.c_void_p(res._ptr), None
    else:
        res = ndarray._empty(src._shape, np.int64)
        y, idx = None, ctypes.c_void_p(res._ptr)
    if src.size:
        _cb.check(_cb.lib.mmp_sort(MMP_CODES[src._dtype], ctypes.c_void_p(src._ptr), y, idx, rows, cols), "sort")
    return res


def sort(a, axis=-1, kind=None, order=None, *, stable=None):
    """Sorted copy along ``axis`` (numpy order, NaN last)."""
    if order is not None:
        raise NotImplementedError("sort(order=...) needs structured dtypes, which are not on the device path")
    src, ax, nd = _rows_last(_asarray(a), axis)
    return _back(_run(src, True), ax, nd)


def argsort(a, axis=-1, kind=None, order=None, *, stable=None):
    """Indices (int64) that sort ``a`` along ``axis``; ties keep their order."""
    if order is not None:
        raise NotImplementedError("argsort(order=...) needs structured dtypes, which are not on the device path")
    src, ax, nd = _rows_last(_asarray(a), axis)
    return _back(_run(src, False), ax, nd)


def msort(a):
    """Sorted copy along the first axis (``sorting.msort``)."""
    return sort(a, axis=0)


def searchsorted(a, v, side="left", sorter=None):
    """Insertion points of ``v`` into the ascending 1-D ``a`` (int64, the
    shape of ``v``; a 0-d array for a scalar ``v``, as the reference)."""
    from . import reductions

    a = _asarray(a)
    if a.ndim != 1:
        raise ValueError("object too deep for desired array")
    if side not in ("left", "right"):
        raise ValueError(f"side must be 'left' or 'right' (got {side!r})")
    vv = v if isinstance(v, ndarray) else _asarray(np.asarray(v))
    dt = np.result_type(a.dtype, vv.dtype)
    a_c = (a if a.dtype == dt else a.astype(dt))._ensure_contiguous()
    v_c = (vv if vv.dtype == dt else vv.astype(dt))._ensure_contiguous()
    s_ptr = None
    if sorter is not None:
        s = _asarray(sorter)
        if s.shape != a.shape:
            raise ValueError("sorter.size must equal a.size")
        if s.dtype.kind not in "iu":
            raise TypeError("sorter must only contain integers")
        if s.size and (int(reductions.min(s).get()) < 0 or int(reductions.max(s).get()) >= a.size):
            raise ValueError("Sorter index out of range.")
        s = (s if s.dtype == np.int64 else s.astype(np.int64))._ensure_contiguous()
        s_ptr = ctypes.c_void_p(s._ptr)
    out = ndarray._empty(v_c._shape, np.int64)
    if v_c.size:
        _cb.check(_cb.lib.mmp_searchsorted(MMP_CODES[dt], ctypes.c_void_p(a_c._ptr if a_c.size else 0), a_c.size,
                                           ctypes.c_void_p(v_c._ptr), v_c.size, 0 if side == "left" else 1,
                                           s_ptr, ctypes.c_void_p(out._ptr)), "searchsorted")
    return out
