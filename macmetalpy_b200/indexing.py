"""Indexing routines (mirrors ``src/macmetalpy/indexing.py:24-410`` and
``math_ops.where``), on the device.

The reference runs each of these with numpy on a host copy.  Here they are
built from the device advanced-indexing primitives (``_advindex``: offset
arrays + ``mmp_gather`` / ``mmp_scatter``, ``mmp_compact_indices``) and
fused elementwise expressions, with numpy's results:

* ``take`` / ``put`` with ``mode`` "raise" (IndexError), "wrap" (modulo) or
  "clip"; ``put`` repeats ``v`` cyclically over the indices;
* ``take_along_axis`` / ``put_along_axis``: numpy's index broadcasting;
* ``putmask`` repeats ``values`` over the array positions (a[i] =
  values[i % len]), ``place`` over the true positions in order;
* ``compress`` / ``extract``: selection by a boolean condition;
* ``nonzero`` / ``flatnonzero`` / ``argwhere``: int64 index arrays;
* ``select`` / ``choose``: fused selects;
* ``unravel_index`` / ``ravel_multi_index``: int64 arithmetic;
* ``fill_diagonal``: a strided view assignment.
"""

from __future__ import annotations

import numbers

import numpy as np

from . import _advindex
from .ndarray import ndarray

__all__ = [
    "take", "take_along_axis", "put", "put_along_axis", "putmask", "place", "compress", "extract",
    "nonzero", "flatnonzero", "argwhere", "select", "choose", "unravel_index", "ravel_multi_index",
    "fill_diagonal", "ix_", "diag_indices", "tril_indices", "triu_indices",
]


def _arr(x) -> ndarray:
    from .creation import asarray

    return x if isinstance(x, ndarray) else asarray(np.asarray(x))


def _norm_axis(axis, nd):
    if not -nd <= axis < nd:
        raise np.exceptions.AxisError(axis, nd)
    return axis % nd


def _moded(idx: ndarray, n: int, mode: str) -> ndarray:
    if mode == "raise":
        return idx
    if n == 0:
        raise IndexError("cannot do a non-empty take from an empty axes.")
    if mode == "wrap":
        return (idx % n)._ensure_contiguous()
    if mode == "clip":
        return idx.clip(0, n - 1)._ensure_contiguous()
    raise ValueError(f"clipmode must be one of 'clip', 'raise', or 'wrap' (got {mode!r})")


def take(a, indices, axis=None, out=None, mode="raise"):
    a = _arr(a)
    scalar = isinstance(indices, (numbers.Integral, np.integer))
    idx = _arr(np.asarray(indices) if scalar else indices)
    if idx.dtype.kind not in "iu":
        raise TypeError("Cannot cast array data from dtype('float64') to dtype('int64') according to the rule 'safe'")
    if axis is None:
        src, ax = a.reshape(-1), 0
    else:
        src, ax = a, _norm_axis(int(axis), a.ndim)
    idx = _moded(idx.astype(np.int64) if idx.dtype != np.int64 else idx, src.shape[ax], mode)
    r = src[(slice(None),) * ax + (idx,)]
    if out is not None:
        out[...] = r
        return out
    return r


def take_along_axis(arr, indices, axis):
    arr, idx = _arr(arr), _arr(indices)
    if axis is None:
        arr, axis = arr.reshape(-1), 0
    ax = _norm_axis(int(axis), arr.ndim)
    if idx.ndim != arr.ndim:
        raise ValueError("`indices` and `arr` must have the same number of dimensions")
    return arr[_along_key(arr, idx, ax)]


def _along_key(arr, idx, ax):
    key = []
    for d in range(arr.ndim):
        if d == ax:
            key.append(idx)
        else:
            shp = [1] * arr.ndim
            shp[d] = arr.shape[d]
            key.append(_arr(np.arange(arr.shape[d], dtype=np.int64).reshape(shp)))
    return tuple(key)


def put_along_axis(arr, indices, values, axis):
    arr, idx = _arr(arr), _arr(indices)
    if axis is None:
        flat = arr.reshape(-1)
        flat[_along_key(flat, idx, 0)] = values
        return None
    ax = _norm_axis(int(axis), arr.ndim)
    arr[_along_key(arr, idx, ax)] = values
    return None


def _cycle(v: ndarray, n: int) -> ndarray:
    """v repeated cyclically to length n (1-D)."""
    v = v.reshape(-1)
    if v.size == n:
        return v._ensure_contiguous()
    pos = _arr(np.arange(n, dtype=np.int64) % max(v.size, 1))
    return v[pos]


def put(a, ind, v, mode="raise"):
    """a.flat[ind] = v, v repeated over the indices."""
    if not isinstance(a, ndarray):
        raise TypeError("put() requires a device array as its first argument")
    flat = a.reshape(-1)
    if not flat._is_c_contiguous() or flat._buffer is not a._buffer:
        raise NotImplementedError("put() on a non-contiguous view is not supported")
    idx = _arr(ind).reshape(-1)
    idx = _moded(idx.astype(np.int64) if idx.dtype != np.int64 else idx, flat.size, mode)
    if idx.size == 0:
        return None
    vals = _cycle(_arr(v).astype(a.dtype) if _arr(v).dtype != a.dtype else _arr(v), idx.size)
    flat[idx] = vals
    return None


def putmask(a, mask, values):
    """a[i] = values[i % len(values)] where mask[i] (numpy's putmask)."""
    mask = _arr(mask)
    if mask.shape != a.shape:
        raise ValueError("putmask: mask and data must be the same size")
    v = _arr(values)
    if v.size == 0:
        return None
    if v.size == 1:
        vv = v.reshape(())
    else:
        vv = _cycle(v, a.size).reshape(a.shape)
    m = mask if mask.dtype == np.bool_ else (mask != 0)
    a[...] = ndarray._select(m, vv, a)
    return None


def place(arr, mask, vals):
    """The k-th true position of ``mask`` gets vals[k % len(vals)]."""
    mask = _arr(mask)
    if mask.size != arr.size:
        raise ValueError("place: mask and data must be the same size")
    pos = _advindex.flatnonzero(mask)
    if pos.size == 0:
        return None
    v = _arr(vals)
    if v.size == 0:
        raise ValueError("Cannot insert from an empty array!")
    flat = arr.reshape(-1)
    flat[pos] = _cycle(v, pos.size)
    return None


def compress(condition, a, axis=None, out=None):
    c = _arr(condition).reshape(-1)
    a = _arr(a)
    if axis is None:
        a, ax = a.reshape(-1), 0
    else:
        ax = _norm_axis(int(axis), a.ndim)
    n = a.shape[ax]
    if c.size > n:
        raise IndexError(f"index {c.size - 1} is out of bounds for axis {ax} with size {n}")
    idx = _advindex.flatnonzero(c)
    r = a[(slice(None),) * ax + (idx,)]
    if out is not None:
        out[...] = r
        return out
    return r


def extract(condition, arr):
    c = _arr(condition).reshape(-1)
    return _arr(arr).reshape(-1)[c != 0 if c.dtype != np.bool_ else c]


def nonzero(a):
    return _advindex.nonzero(_arr(a))


def flatnonzero(a):
    return _advindex.flatnonzero(_arr(a))


def argwhere(a):
    a = _arr(a)
    if a.ndim == 0:
        return _arr(np.zeros((int(bool(a.get())), 0), dtype=np.int64))
    idx = _advindex.nonzero(a)
    out = ndarray._empty((idx[0].size, a.ndim), np.int64)
    for d, ix in enumerate(idx):
        out[:, d] = ix
    return out


def select(condlist, choicelist, default=0):
    if len(condlist) != len(choicelist):
        raise ValueError("list of cases must be same length as list of conditions")
    if not condlist:
        raise ValueError("select with an empty condition list is not possible")
    r = default
    for c, v in zip(reversed(condlist), reversed(choicelist)):
        c = _arr(c)
        if c.dtype != np.bool_:
            raise TypeError(f"invalid entry in condlist: should be boolean ndarray")
        r = ndarray._select(c, v, r)
    return r if isinstance(r, ndarray) else _arr(np.asarray(r))


def choose(a, choices, out=None, mode="raise"):
    a = _arr(a)
    n = len(choices)
    if mode == "raise":
        from . import reductions

        if a.size and (int(reductions.min(a).get()) < 0 or int(reductions.max(a).get()) >= n):
            raise ValueError("invalid entry in choice array")
        idx = a
    elif mode == "wrap":
        idx = a % n
    elif mode == "clip":
        idx = a.clip(0, n - 1)
    else:
        raise ValueError(f"clipmode must be one of 'clip', 'raise', or 'wrap' (got {mode!r})")
    r = choices[n - 1]
    for k in range(n - 2, -1, -1):
        r = ndarray._select(idx == k, choices[k], r)
    r = r if isinstance(r, ndarray) else _arr(np.asarray(r))
    if out is not None:
        out[...] = r
        return out
    return r


def unravel_index(indices, shape, order="C"):
    if order != "C":
        raise NotImplementedError("unravel_index(order='F') is not supported")
    idx = _arr(indices)
    size = int(np.prod(shape))
    from . import reductions

    if idx.size and (int(reductions.min(idx).get()) < 0 or int(reductions.max(idx).get()) >= size):
        raise ValueError(f"index {int(reductions.max(idx).get())} is out of bounds for array with size {size}")
    idx = idx.astype(np.int64) if idx.dtype != np.int64 else idx
    return tuple(x._ensure_contiguous() if isinstance(x, ndarray) else x
                 for x in _advindex.unravel(idx, tuple(shape)))


def ravel_multi_index(multi_index, dims, mode="raise", order="C"):
    if order != "C":
        raise NotImplementedError("ravel_multi_index(order='F') is not supported")
    from . import reductions

    parts = [_arr(m) for m in multi_index]
    if len(parts) != len(dims):
        raise ValueError(f"parameter multi_index must be a sequence of length {len(dims)}")
    r = None
    for p, d in zip(parts, dims):
        p = p.astype(np.int64) if p.dtype != np.int64 else p
        if mode == "raise":
            if p.size and (int(reductions.min(p).get()) < 0 or int(reductions.max(p).get()) >= d):
                raise ValueError("invalid entry in coordinates array")
        elif mode == "wrap":
            p = p % d
        elif mode == "clip":
            p = p.clip(0, d - 1)
        r = p if r is None else r * d + p
    return r._ensure_contiguous()


def fill_diagonal(a, val, wrap=False):
    if a.ndim < 2:
        raise ValueError("array must be at least 2-d")
    if a.ndim > 2 and len(set(a.shape)) != 1:
        raise ValueError("All dimensions of input must be of equal length")
    n = min(a.shape)
    step = sum(a._strides)
    if a.ndim == 2 and wrap and a.shape[0] > a.shape[1]:
        # numpy's wrap: flat C-order positions 0, C+1, 2(C+1), ... below R*C
        R, C = a.shape
        pos = np.arange(0, R * C, C + 1, dtype=np.int64)
        offs = (pos // C) * a._strides[0] + (pos % C) * a._strides[1] + a._offset
        flat = ndarray._from_buffer(a._buffer, (a._buffer.nbytes // a.dtype.itemsize,), a.dtype)
        flat[_arr(offs)] = val
        return None
    diag = ndarray._from_buffer(a._buffer, (n,), a.dtype, strides=(step,), offset=a._offset, base=a)
    diag[...] = val
    return None


def ix_(*args):
    out = []
    nd = len(args)
    for k, x in enumerate(args):
        x = _arr(x)
        if x.ndim != 1:
            raise ValueError("Cross index must be 1 dimensional")
        if x.dtype == np.bool_:
            x = _advindex.flatnonzero(x)
        shp = [1] * nd
        shp[k] = x.size
        out.append(x.reshape(shp))
    return tuple(out)


def diag_indices(n, ndim=2):
    i = _arr(np.arange(n, dtype=np.int64))
    return (i,) * ndim


def tril_indices(n, k=0, m=None):
    return tuple(_arr(x) for x in np.tril_indices(n, k, m))


def triu_indices(n, k=0, m=None):
    return tuple(_arr(x) for x in np.triu_indices(n, k, m))
