"""Advanced (integer- and boolean-array) indexing on the device.

The reference answers every advanced key with numpy on a host copy
(``ndarray.py:874-957``).  Here a key is turned into one int64 array of
element offsets with numpy's rules, and ``mmp_gather`` / ``mmp_scatter``
move the elements:

* a boolean array index is replaced by its nonzero index arrays (device
  compaction: scan of the mask + ``mmp_compact_indices``), and must match
  the dimensions it covers;
* integer scalars count as advanced indices once any array index is present;
* all advanced indices broadcast together to a shape B; when they are
  adjacent in the key, B takes their place in the result, otherwise B comes
  first (numpy's rule); slices and ``None`` keep their axes;
* an index outside [-size, size) raises numpy's IndexError before any
  element moves; negative indices count from the end.

The offsets are one fused elementwise expression over small per-axis
vectors and the (broadcast) index arrays.  ``a[mask]`` with a full-shape
mask on a contiguous array skips the offset build: the compacted positions
are the offsets.  ``a[mask] = scalar`` with a full-shape mask is a fused
in-place select (no compaction).  An assignment through integer arrays
that name one element several times keeps the last value, as numpy does:
the offsets are sorted stably on the device (``mmp_sort``) and only the last
of each run of equal offsets is written.
"""

from __future__ import annotations

import ctypes
import math
import numbers

import numpy as np

from . import _cuda_backend as _cb
from ._broadcasting import broadcast_shapes
from ._dtypes import MMP_CODES


def _nd():
    from .ndarray import ndarray
    return ndarray


def _upload(x):
    from .creation import asarray
    return asarray(np.asarray(x))


def _iota(n: int):
    """int64 0..n-1 on the device."""
    return _upload(np.arange(n, dtype=np.int64))


def flatnonzero(mask):
    """int64 positions (C order) of the nonzero entries of ``mask``."""
    from . import reductions
    ndarray = _nd()
    m = mask if mask.dtype == np.bool_ else (mask != 0)
    m = m.reshape(-1)._ensure_contiguous()
    n = m.size
    if n == 0:
        return ndarray._empty((0,), np.int64)
    incl = reductions.cumsum(m)
    count = int(incl[n - 1].get())
    out = ndarray._empty((count,), np.int64)
    if count:
        _cb.check(_cb.lib.mmp_compact_indices(ctypes.c_void_p(m._ptr), ctypes.c_void_p(incl._ptr), n, count,
                                              ctypes.c_void_p(out._ptr)), "nonzero")
    return out


def unravel(flat, shape):
    """Per-dimension index arrays of C-order flat positions."""
    out = []
    rest = 1
    for s in reversed(shape):
        out.append((flat // rest) % s if len(shape) > 1 else flat)
        rest *= s
    return tuple(reversed(out))


def nonzero(a):
    if a.ndim == 0:
        raise ValueError("Calling nonzero on 0d arrays is not allowed. Use np.atleast_1d(scalar).nonzero() instead.")
    flat = flatnonzero(a)
    return tuple(x._ensure_contiguous() if hasattr(x, "_ensure_contiguous") else x for x in unravel(flat, a.shape))


def _is_adv(k) -> bool:
    ndarray = _nd()
    if isinstance(k, ndarray):
        return True
    if isinstance(k, (list, np.ndarray)):
        return True
    return False


def is_advanced(key) -> bool:
    if not isinstance(key, tuple):
        key = (key,)
    return any(_is_adv(k) or isinstance(k, (bool, np.bool_)) for k in key)


def _normalise(a, key):
    """Expand the key to one entry per consumed dimension (plus None):
    ints, slices, None, and ("arr", int64 device array, dim) entries."""
    ndarray = _nd()
    if not isinstance(key, tuple):
        key = (key,)
    items = []
    for k in key:
        if k is None or k is Ellipsis or isinstance(k, slice):
            items.append(k)
        elif isinstance(k, (bool, np.bool_)):
            raise NotImplementedError("a scalar boolean index is not supported on the device path")
        elif isinstance(k, (numbers.Integral, np.integer)):
            items.append(int(k))
        else:
            arr = k if isinstance(k, ndarray) else _upload(k)
            if arr.dtype == np.bool_:
                items.append(("bool", arr))
            elif arr.dtype.kind in "iu":
                items.append(("int", arr))
            else:
                raise IndexError("arrays used as indices must be of integer (or boolean) type")
    if sum(1 for k in items if k is Ellipsis) > 1:
        raise IndexError("an index can only have a single ellipsis ('...')")
    used = sum(1 if not isinstance(k, tuple) else (k[1].ndim if k[0] == "bool" else 1)
               for k in items if k is not None and k is not Ellipsis)
    if used > a.ndim:
        raise IndexError(f"too many indices for array: array is {a.ndim}-dimensional, but {used} were indexed")
    out = []
    dim = 0
    for k in items:
        if k is Ellipsis:
            for _ in range(a.ndim - used):
                out.append((slice(None), dim))
                dim += 1
        elif k is None:
            out.append((None, dim))
        elif isinstance(k, tuple) and k[0] == "bool":
            m = k[1]
            if m.ndim == 0:
                raise NotImplementedError("a 0-d boolean index is not supported on the device path")
            for j, s in enumerate(m.shape):
                if a.shape[dim + j] != s:
                    raise IndexError(f"boolean index did not match indexed array along axis {dim + j}; size of "
                                     f"axis is {a.shape[dim + j]} but size of corresponding boolean axis is {s}")
            for j, ix in enumerate(nonzero(m)):
                out.append((("arr", ix), dim + j))
            dim += m.ndim
        elif isinstance(k, tuple):
            out.append((("arr", k[1]), dim))
            dim += 1
        else:
            out.append((k, dim))
            dim += 1
    while dim < a.ndim:
        out.append((slice(None), dim))
        dim += 1
    return out


def _check_range(idx, size, axis):
    from . import reductions
    if idx.size == 0:
        return
    hi = int(reductions.max(idx).get())
    lo = int(reductions.min(idx).get())
    if hi >= size:
        raise IndexError(f"index {hi} is out of bounds for axis {axis} with size {size}")
    if lo < -size:
        raise IndexError(f"index {lo} is out of bounds for axis {axis} with size {size}")


def offsets(a, key):
    """(int64 offsets array of the selection, selection shape)."""
    ndarray = _nd()
    items = _normalise(a, key)
    adv_pos = [i for i, (k, _) in enumerate(items) if isinstance(k, (int, tuple))]
    has_arr = any(isinstance(k, tuple) for k, _ in items)
    if not has_arr:
        raise AssertionError("offsets() needs an array index")
    adv_arrays = [k[1] for k, _ in items if isinstance(k, tuple)]
    B = broadcast_shapes(*[x.shape for x in adv_arrays]) if adv_arrays else ()
    adjacent = adv_pos == list(range(adv_pos[0], adv_pos[-1] + 1))
    # output layout: basic axes (slice / None) and the block B
    basic = [(i, k) for i, (k, _) in enumerate(items) if not isinstance(k, (int, tuple))]
    layout = []  # entries: ("b", item index, length) or ("B",)
    if adjacent:
        for i, k in basic:
            if i < adv_pos[0]:
                layout.append(("b", i))
        layout.append(("B",))
        for i, k in basic:
            if i > adv_pos[-1]:
                layout.append(("b", i))
    else:
        layout.append(("B",))
        for i, k in basic:
            layout.append(("b", i))
    lengths = {}
    for i, (k, d) in enumerate(items):
        if isinstance(k, slice):
            start, stop, step = k.indices(a.shape[d])
            lengths[i] = (len(range(start, stop, step)), start, step)
        elif k is None:
            lengths[i] = (1, 0, 0)
    out_shape = []
    axis_of = {}
    b0 = None
    for ent in layout:
        if ent[0] == "B":
            b0 = len(out_shape)
            out_shape.extend(B)
        else:
            axis_of[ent[1]] = len(out_shape)
            out_shape.append(lengths[ent[1]][0])
    out_shape = tuple(out_shape)
    nd = len(out_shape)
    expr = None
    const = a._offset
    for i, (k, d) in enumerate(items):
        st = a._strides[d] if d < a.ndim else 0
        if k is None:
            continue
        if isinstance(k, slice):
            L, start, step = lengths[i]
            const += start * st
            if L > 1 and step * st != 0:
                shp = [1] * nd
                shp[axis_of[i]] = L
                term = _iota(L).reshape(shp) * (step * st)
                expr = term if expr is None else expr + term
        elif isinstance(k, int):
            size = a.shape[d]
            j = k + size if k < 0 else k
            if not 0 <= j < size:
                raise IndexError(f"index {k} is out of bounds for axis {d} with size {size}")
            const += j * st
        else:
            idx = k[1]
            size = a.shape[d]
            _check_range(idx, size, d)
            idx = idx if idx.dtype == np.int64 else idx.astype(np.int64)
            w = ndarray._select(idx < 0, idx + size, idx)
            shp = [1] * nd
            sub = (1,) * (len(B) - idx.ndim) + tuple(idx.shape)
            shp[b0:b0 + len(B)] = sub
            term = w.reshape(shp) * st
            expr = term if expr is None else expr + term
    n = math.prod(out_shape)
    off = ndarray._empty(out_shape, np.int64)
    if n:
        if expr is None:
            off[...] = const
        else:
            off[...] = expr + const
    return off, out_shape


def _limit(a) -> int:
    return a._buffer.nbytes // a.dtype.itemsize


def _full_mask(a, key):
    """The bool mask when ``key`` is one mask of ``a``'s full shape."""
    ndarray = _nd()
    k = key[0] if isinstance(key, tuple) and len(key) == 1 else key
    if isinstance(k, (list, np.ndarray)):
        k = _upload(k) if np.asarray(k).dtype == np.bool_ else None
    if isinstance(k, ndarray) and k.dtype == np.bool_ and k.shape == a.shape and a.ndim > 0:
        return k
    return None


def getitem(a, key):
    ndarray = _nd()
    mask = _full_mask(a, key)
    if mask is not None and a._is_c_contiguous():
        off = flatnonzero(mask)
        if a._offset:
            off = (off + a._offset)._ensure_contiguous()
        shape = off.shape
    else:
        off, shape = offsets(a, key)
    out = ndarray._empty(shape, a.dtype)
    if out.size:
        _cb.check(_cb.lib.mmp_gather(MMP_CODES[a.dtype], ctypes.c_void_p(a._buffer.ptr), _limit(a),
                                     ctypes.c_void_p(off._ptr), out.size, ctypes.c_void_p(out._ptr)), "gather")
    return out


def _last_wins(off, vals):
    """Offsets / values with every repeated offset reduced to its last
    occurrence (stable device argsort of the offsets)."""
    from . import sorting
    ndarray = _nd()
    off = off.reshape(-1)._ensure_contiguous()
    vals = vals.reshape(-1)._ensure_contiguous()
    n = off.size
    if n <= 1:
        return off, vals
    perm = sorting.argsort(off)
    so = off[perm]
    keep = ndarray._empty((n,), np.bool_)
    keep[: n - 1] = so[: n - 1] != so[1:]
    keep[n - 1] = True
    sel = flatnonzero(keep)
    if sel.size == n:
        return off, vals
    return so[sel], vals[perm[sel]]


def _has_int_array(a, key):
    keys = key if isinstance(key, tuple) else (key,)
    ndarray = _nd()
    for k in keys:
        if isinstance(k, (ndarray, list, np.ndarray)):
            dt = k.dtype if isinstance(k, (ndarray, np.ndarray)) else np.asarray(k).dtype
            if dt != np.bool_:
                return True
    return False


def setitem(a, key, value):
    ndarray = _nd()
    mask = _full_mask(a, key)
    is_scalar = isinstance(value, (numbers.Number, np.generic)) or (isinstance(value, np.ndarray) and value.ndim == 0)
    if mask is not None and is_scalar:
        a[...] = ndarray._select(mask, np.asarray(value).astype(a.dtype)[()], a)
        return
    if mask is not None and a._is_c_contiguous():
        off = flatnonzero(mask)
        if a._offset:
            off = (off + a._offset)._ensure_contiguous()
        shape = off.shape
    else:
        off, shape = offsets(a, key)
    if off.size == 0:
        return
    vals = ndarray._empty(shape, a.dtype)
    vals[...] = value
    if _has_int_array(a, key):  # integer arrays may name an element twice
        off, vals = _last_wins(off, vals)
    _cb.check(_cb.lib.mmp_scatter(MMP_CODES[a.dtype], ctypes.c_void_p(a._buffer.ptr), _limit(a),
                                  ctypes.c_void_p(off._ptr), off.size, ctypes.c_void_p(vals._ptr)), "scatter")
