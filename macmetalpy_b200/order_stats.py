"""Order statistics, unique, lexsort and partition on the device.

The reference runs all of these through numpy on the host:
``reductions.median/percentile/quantile`` (``reductions.py:627-820``),
``nan_ops.nanmedian/nanpercentile/nanquantile`` (``nan_ops.py:435-800``),
``sorting.unique/lexsort/partition/argpartition/unique_*``
(``sorting.py:200-370``).  Here every function sorts on the device (the
radix sort of :mod:`sorting`) and picks and combines the order statistics
with device ops.  Results are numpy's, bit for bit where numpy's arithmetic
is reproduced:

* ``median``: the middle element, or numpy's mean of the two middle ones
  ((lo + hi) / 2 in the float type, float16 through float32, integers in
  float64); NaN for a slice that holds a NaN (NaN sorts last).
* ``percentile`` / ``quantile`` (method ``'linear'``): numpy's virtual index
  (n - 1) q, its floor and fraction, computed on the host as numpy computes
  them (they depend on n and q only, in the dtype numpy gives q), the two
  order statistics picked from the sorted rows, then numpy's two-sided
  interpolation: a + (b - a) t, or b - (b - a)(1 - t) where t >= 0.5.
* the nan-versions: the same per row over its non-NaN values (a count per
  row, indices and fractions computed on the device), NaN for all-NaN rows.
* ``unique``: stable argsort, run starts (NaNs equal, as numpy's
  ``equal_nan=True``), compaction; first indices, inverse and counts on
  request.  With ``axis``: rows ordered lexicographically by ``lexsort``.
* ``lexsort``: stable argsorts from the first (least significant) key to
  the last.
* ``partition`` / ``argpartition``: the sorted array and the stable argsort.
  Both meet numpy's contract: the k-th element in its sorted place, nothing
  larger before it, nothing smaller after it.  numpy leaves the order inside
  the two sides unspecified, so the arrays themselves may differ from
  numpy's introselect output.
"""

from __future__ import annotations

import math
from collections import namedtuple

import numpy as np

from . import reductions, sorting
from .ndarray import ndarray

__all__ = ["median", "percentile", "quantile", "nanmedian", "nanpercentile", "nanquantile", "unique",
           "unique_all", "unique_counts", "unique_inverse", "unique_values", "lexsort", "partition",
           "argpartition"]


def _asarray(a) -> ndarray:
    if isinstance(a, ndarray):
        return a
    from .creation import asarray

    return asarray(np.asarray(a))


def _out(r: ndarray, out):
    if out is None:
        return r
    out[...] = r
    return out


def _axes_last(a: ndarray, axis):
    """(array with the reduced axes merged into the last one, kept shape,
    keepdims shape).  ``axis=None`` reduces everything."""
    nd = a.ndim
    if axis is None:
        return a.reshape(-1), (), (1,) * nd
    axes = (axis,) if isinstance(axis, (int, np.integer)) else tuple(axis)
    axes = np.lib.array_utils.normalize_axis_tuple(axes, nd)
    rest = [i for i in range(nd) if i not in axes]
    order = rest + sorted(axes)
    b = a.transpose(order) if order != list(range(nd)) else a
    kept = tuple(a.shape[i] for i in rest)
    n = math.prod(a.shape[i] for i in axes)
    kshape = tuple(1 if i in axes else a.shape[i] for i in range(nd))
    return b.reshape(kept + (n,)), kept, kshape


def _sorted_rows(a: ndarray, axis):
    b, kept, kshape = _axes_last(a, axis)
    return sorting.sort(b, axis=-1), kept, kshape


def _nan_of(dt):
    return np.dtype(dt).type(np.nan)


def _median_dtype(dt) -> np.dtype:
    return np.median(np.zeros(1, dtype=dt)).dtype


def _mid_mean(lo: ndarray, hi: ndarray, dt: np.dtype) -> ndarray:
    """numpy's mean of the two middle values, in numpy's types: the float
    type itself, float16 through float32, integers and bool in float64."""
    if dt == np.float16:
        return ((lo.astype(np.float32) + hi.astype(np.float32)) / np.float32(2)).astype(np.float16)
    if dt.kind == "f":
        return (lo + hi) / dt.type(2)
    return (lo.astype(np.float64) + hi.astype(np.float64)) / np.float64(2)


def _pick(s: ndarray, idx: ndarray) -> ndarray:
    """s[..., idx[...]] along the last axis (one index per row)."""
    from .indexing import take_along_axis

    return take_along_axis(s, idx.reshape(idx.shape + (1,)), axis=-1).reshape(idx.shape)


def _full(shape, value, dt) -> ndarray:
    from .creation import full

    return full(shape, value, dtype=dt)


# ---------------------------------------------------------------- median
def median(a, axis=None, out=None, overwrite_input=False, keepdims=False):
    """Median along ``axis`` (numpy's ``median``; NaN where a slice holds NaN)."""
    from .logic_ops import isnan
    from .math_ops import where

    a = _asarray(a)
    dt = a.dtype
    odt = _median_dtype(dt)
    s, kept, kshape = _sorted_rows(a, axis)
    n = s.shape[-1]
    if n == 0:
        r = _full(kept, np.nan, odt)
    else:
        if n % 2:
            r = s[..., n // 2].astype(odt)
        else:
            r = _mid_mean(s[..., n // 2 - 1], s[..., n // 2], dt)
        if dt.kind == "f":
            last = s[..., n - 1]
            r = where(isnan(last), last, r)
    if keepdims:
        r = r.reshape(kshape)
    return _out(r, out)


def nanmedian(a, axis=None, out=None, overwrite_input=False, keepdims=False):
    """Median of the non-NaN values (numpy's ``nanmedian``; NaN for all-NaN
    slices)."""
    from .logic_ops import isnan, logical_not
    from .math_ops import where

    a = _asarray(a)
    dt = a.dtype
    if dt.kind != "f":
        return median(a, axis=axis, out=out, keepdims=keepdims)
    s, kept, kshape = _sorted_rows(a, axis)
    n = s.shape[-1]
    if n == 0:
        r = _full(kept, np.nan, dt)
    else:
        c = reductions.sum(logical_not(isnan(s)), axis=-1)  # non-NaN values per row, sorted first
        h = c // 2
        odd = (c % 2) == 1
        lo_i = where(odd, h, where(h > 0, h - 1, 0))
        hi_i = where(h < n, h, n - 1)
        lo, hi = _pick(s, lo_i), _pick(s, hi_i)
        r = where(odd, lo, _mid_mean(lo, hi, dt))
        r = where(c == 0, _nan_of(dt), r)
    if keepdims:
        r = r.reshape(kshape)
    return _out(r, out)


# ---------------------------------------------------------------- quantiles
def _q_percentile(q, dt):
    """q / 100 in the dtype numpy's ``percentile`` gives it."""
    if isinstance(q, ndarray):
        q = q.get()
    qa = np.asanyarray(np.true_divide(q, dt.type(100) if dt.kind == "f" else 100))
    if qa.size and not (np.all(qa >= 0) and np.all(qa <= 1)):
        raise ValueError("Percentiles must be in the range [0, 100]")
    return qa


def _q_quantile(q, dt):
    """q in the dtype numpy's ``quantile`` gives it (a Python scalar takes
    the array's float type)."""
    if isinstance(q, ndarray):
        q = q.get()
    if isinstance(q, (int, float)) and dt.kind == "f":
        qa = np.asanyarray(q, dtype=dt)
    else:
        qa = np.asanyarray(q)
    if qa.size and not (np.all(qa >= 0) and np.all(qa <= 1)):
        raise ValueError("Quantiles must be in the range [0, 1]")
    return qa


def _lerp(lo: ndarray, hi: ndarray, t):
    """numpy's two-sided linear interpolation for one scalar weight t."""
    diff = hi - lo
    if t >= 0.5:
        return hi - diff * (1 - t)
    return lo + diff * t


def _stack(parts, qshape, kept, dt) -> ndarray:
    if len(qshape) == 0:
        return parts[0]
    res = ndarray._empty(tuple(qshape) + tuple(kept), np.dtype(dt))
    for j, p in enumerate(parts):
        res[np.unravel_index(j, qshape)] = p
    return res


def _quantile_sorted(s: ndarray, qa: np.ndarray, dt: np.dtype):
    """numpy's 'linear' quantiles of every row of the sorted ``s``."""
    from .logic_ops import isnan
    from .math_ops import where

    n = s.shape[-1]
    vi = np.asanyarray((n - 1) * qa)  # numpy's virtual index, in numpy's dtype
    parts = []
    if np.issubdtype(vi.dtype, np.integer):  # integral q: no interpolation
        for v in vi.reshape(-1):
            r = s[..., int(v)].copy()
            if dt.kind == "f":
                last = s[..., n - 1]
                r = where(isnan(last), last, r)
            parts.append(r)
        return parts
    # floor / next / fraction exactly as numpy's _get_indexes and _get_gamma
    prev = np.asanyarray(np.floor(vi))
    nxt = np.asanyarray(prev + 1)
    above = vi >= n - 1
    prev[above] = -1
    nxt[above] = -1
    below = vi < 0
    prev[below] = 0
    nxt[below] = 0
    nanv = np.isnan(vi)
    prev[nanv] = -1
    nxt[nanv] = -1
    prev = prev.astype(np.intp)
    nxt = nxt.astype(np.intp)
    gamma = np.asanyarray(vi - prev, dtype=vi.dtype)
    for pv, nv, g in zip(prev.reshape(-1), nxt.reshape(-1), gamma.reshape(-1)):
        r = _lerp(s[..., int(pv) % n], s[..., int(nv) % n], g)
        if dt.kind == "f":
            last = s[..., n - 1]
            r = where(isnan(last), last, r)
        parts.append(r)
    return parts


def _quantile(a, qa, axis, out, keepdims):
    a = _asarray(a)
    dt = a.dtype
    s, kept, kshape = _sorted_rows(a, axis)
    n = s.shape[-1]
    if n == 0:
        raise IndexError("index -1 is out of bounds for axis 0 with size 0")
    parts = _quantile_sorted(s, qa, dt)
    r = _stack(parts, qa.shape, kept, parts[0].dtype)
    if keepdims:
        r = r.reshape(tuple(qa.shape) + kshape)
    return _out(r, out)


def _check_method(method):
    if method != "linear":
        raise NotImplementedError(f"method={method!r}: only numpy's default 'linear' is on the device path")


def percentile(a, q, axis=None, out=None, overwrite_input=False, method="linear", keepdims=False):
    """q-th percentiles along ``axis`` (numpy's ``percentile``, method 'linear')."""
    _check_method(method)
    a = _asarray(a)
    return _quantile(a, _q_percentile(q, a.dtype), axis, out, keepdims)


def quantile(a, q, axis=None, out=None, overwrite_input=False, method="linear", keepdims=False):
    """q-th quantiles along ``axis`` (numpy's ``quantile``, method 'linear')."""
    _check_method(method)
    a = _asarray(a)
    return _quantile(a, _q_quantile(q, a.dtype), axis, out, keepdims)


def _nanquantile(a, qa, axis, out, keepdims):
    from .logic_ops import isnan, logical_not
    from .math_ops import floor, where

    dt = a.dtype
    s, kept, kshape = _sorted_rows(a, axis)
    n = s.shape[-1]
    if n == 0:
        parts = [_full(kept, np.nan, np.result_type(dt, qa.dtype)) for _ in range(max(qa.size, 1))]
    else:
        c = reductions.sum(logical_not(isnan(s)), axis=-1)  # non-NaN values per row, sorted first
        vdt = np.asanyarray((1 - 1) * qa).dtype  # numpy's virtual-index dtype for this q
        cm1 = (c - 1).astype(vdt)
        parts = []
        for qv in qa.reshape(-1):
            vi = cm1 * vdt.type(qv)
            above = vi >= cm1  # numpy compares with the count - 1 in vi's dtype
            below = vi < 0
            fl = floor(vi)
            prev = where(above, c - 1, where(below, 0, fl.astype(np.int64)))
            nxt = where(above, c - 1, where(below, 0, fl.astype(np.int64) + 1))
            # numpy's fraction: vi minus the substituted index (-1 above, 0
            # below) in float64, then in vi's dtype
            sub = where(above, -1, where(below, 0, prev))
            gamma = (vi.astype(np.float64) - sub.astype(np.float64)).astype(vdt)
            prev = where(prev < 0, 0, prev)
            nxt = where(nxt < 0, 0, where(nxt > n - 1, n - 1, nxt))
            lo, hi = _pick(s, prev), _pick(s, nxt)
            diff = hi - lo
            r = where(gamma >= 0.5, hi - diff * (1 - gamma), lo + diff * gamma)
            r = where(c == 0, _nan_of(r.dtype), r)
            parts.append(r)
    r = _stack(parts, qa.shape, kept, parts[0].dtype)
    if keepdims:
        r = r.reshape(tuple(qa.shape) + kshape)
    return _out(r, out)


def nanpercentile(a, q, axis=None, out=None, overwrite_input=False, method="linear", keepdims=False):
    """q-th percentiles of the non-NaN values (numpy's ``nanpercentile``)."""
    _check_method(method)
    a = _asarray(a)
    if a.dtype.kind != "f":
        return percentile(a, q, axis=axis, out=out, keepdims=keepdims)
    return _nanquantile(a, _q_percentile(q, a.dtype), axis, out, keepdims)


def nanquantile(a, q, axis=None, out=None, overwrite_input=False, method="linear", keepdims=False):
    """q-th quantiles of the non-NaN values (numpy's ``nanquantile``)."""
    _check_method(method)
    a = _asarray(a)
    if a.dtype.kind != "f":
        return quantile(a, q, axis=axis, out=out, keepdims=keepdims)
    return _nanquantile(a, _q_quantile(q, a.dtype), axis, out, keepdims)


# ---------------------------------------------------------------- unique
def _run_starts(s: ndarray, equal_nan: bool) -> ndarray:
    """bool flags: s[i] starts a run of equal values (NaNs equal when
    ``equal_nan``)."""
    from .creation import ones
    from .logic_ops import isnan, logical_and, logical_not

    n = s.shape[0]
    f = ones((n,), dtype=np.bool_)
    if n > 1:
        d = s[1:] != s[:-1]
        if equal_nan and s.dtype.kind == "f":
            d = logical_and(d, logical_not(logical_and(isnan(s[1:]), isnan(s[:-1]))))
        f[1:] = d
    return f


def _unique_flat(a: ndarray, return_index, return_inverse, return_counts, equal_nan):
    from .indexing import flatnonzero, take

    x = a.reshape(-1)
    n = x.size
    i64 = np.dtype(np.int64)
    if n == 0:
        empty = ndarray._empty((0,), i64)
        res = [x.copy()]
        if return_index:
            res.append(empty)
        if return_inverse:
            res.append(ndarray._empty(a.shape, i64))
        if return_counts:
            res.append(ndarray._empty((0,), i64))
        return res
    perm = sorting.argsort(x)
    s = take(x, perm)
    f = _run_starts(s, equal_nan)
    starts = flatnonzero(f)
    res = [take(s, starts)]
    if return_index:
        res.append(take(perm, starts))
    if return_inverse:
        inv = ndarray._empty((n,), i64)
        inv[perm] = reductions.cumsum(f) - 1
        res.append(inv.reshape(a.shape))
    if return_counts:
        k = starts.shape[0]
        counts = ndarray._empty((k,), i64)
        if k > 1:
            counts[:-1] = starts[1:] - starts[:-1]
        counts[k - 1:] = n - starts[k - 1:]
        res.append(counts)
    return res


def _unique_axis(a: ndarray, axis, return_index, return_inverse, return_counts):
    from .indexing import flatnonzero, take

    nd = a.ndim
    ax = int(np.lib.array_utils.normalize_axis_index(axis, nd))
    moved = a.swapaxes(0, ax) if ax else a
    m = moved.shape[0]
    inner = moved.shape[1:]
    rows = moved.reshape(m, -1)
    w = rows.shape[1]
    i64 = np.dtype(np.int64)
    if m == 0 or w == 0:
        raise ValueError("unique along an axis needs non-empty rows on the device path")
    perm = lexsort([rows[:, j] for j in range(w - 1, -1, -1)])  # column 0 most significant
    s = take(rows, perm, axis=0)
    from .creation import ones

    f = ones((m,), dtype=np.bool_)
    if m > 1:
        f[1:] = reductions.any(s[1:] != s[:-1], axis=1)
    starts = flatnonzero(f)
    vals = take(s, starts, axis=0).reshape((starts.shape[0],) + inner)
    vals = vals.swapaxes(0, ax) if ax else vals
    res = [vals.copy()]
    if return_index:
        res.append(take(perm, starts))
    if return_inverse:
        inv = ndarray._empty((m,), i64)
        inv[perm] = reductions.cumsum(f) - 1
        res.append(inv)
    if return_counts:
        k = starts.shape[0]
        counts = ndarray._empty((k,), i64)
        if k > 1:
            counts[:-1] = starts[1:] - starts[:-1]
        counts[k - 1:] = m - starts[k - 1:]
        res.append(counts)
    return res


def unique(ar, return_index=False, return_inverse=False, return_counts=False, axis=None, equal_nan=True, *,
           sorted=True):
    """Sorted unique values (numpy's ``unique``); first indices, inverse
    (the input's shape) and counts on request."""
    a = _asarray(ar)
    if axis is None:
        res = _unique_flat(a, return_index, return_inverse, return_counts, equal_nan)
    else:
        res = _unique_axis(a, axis, return_index, return_inverse, return_counts)
    return res[0] if len(res) == 1 else tuple(res)


UniqueAllResult = namedtuple("UniqueAllResult", ["values", "indices", "inverse_indices", "counts"])
UniqueCountsResult = namedtuple("UniqueCountsResult", ["values", "counts"])
UniqueInverseResult = namedtuple("UniqueInverseResult", ["values", "inverse_indices"])


def unique_all(a):
    """values, first indices, inverse indices and counts (``sorting.unique_all``)."""
    return UniqueAllResult(*unique(a, return_index=True, return_inverse=True, return_counts=True))


def unique_counts(a):
    """values and counts (``sorting.unique_counts``)."""
    return UniqueCountsResult(*unique(a, return_counts=True))


def unique_inverse(a):
    """values and inverse indices (``sorting.unique_inverse``)."""
    return UniqueInverseResult(*unique(a, return_inverse=True))


def unique_values(a):
    """sorted unique values (``sorting.unique_values``)."""
    return unique(a)


# ---------------------------------------------------------------- lexsort / partition
def lexsort(keys, axis=-1):
    """Indirect stable sort by several keys, the last one primary (numpy's
    ``lexsort``): int64 indices along ``axis``."""
    from .indexing import take_along_axis

    if isinstance(keys, ndarray):
        ks = [keys[i] for i in range(keys.shape[0])]
    else:
        ks = [_asarray(k) for k in keys]
    if not ks:
        raise TypeError("need sequence of keys with len > 0 in lexsort")
    shape = ks[0].shape
    for k in ks:
        if k.shape != shape:
            raise ValueError("all keys need to be the same shape")
    perm = sorting.argsort(ks[0], axis=axis)
    for k in ks[1:]:
        kp = take_along_axis(k, perm, axis=axis)
        perm = take_along_axis(perm, sorting.argsort(kp, axis=axis), axis=axis)
    return perm


def _check_kth(a: ndarray, kth, axis):
    n = a.size if axis is None else a.shape[int(np.lib.array_utils.normalize_axis_index(axis, a.ndim))]
    for k in np.atleast_1d(np.asarray(kth)).reshape(-1):
        if not -n <= int(k) < n:
            raise ValueError(f"kth(={int(k)}) out of bounds ({n})")


def partition(a, kth, axis=-1, kind="introselect", order=None):
    """A partitioned copy: the sorted array along ``axis`` (see the module
    notes on numpy's unspecified order inside the two sides)."""
    a = _asarray(a)
    _check_kth(a, kth, axis)
    return sorting.sort(a, axis=axis)


def argpartition(a, kth, axis=-1, kind="introselect", order=None):
    """Indices that partition ``a``: the stable argsort along ``axis``."""
    a = _asarray(a)
    _check_kth(a, kth, axis)
    return sorting.argsort(a, axis=axis)
