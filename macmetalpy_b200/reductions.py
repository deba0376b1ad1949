"""Reductions and scans (mirrors ``src/macmetalpy/reductions.py``).

Same public functions and keywords as the reference (``sum`` ``:74``,
``mean`` ``:116``, ``max``/``min`` ``:166,207``, ``argmax``/``argmin``
``:381,421``, ``std``/``var`` ``:461,525``, ``prod`` ``:587``,
``cumsum``/``cumprod`` ``:661,684``), but every size runs on the GPU:

* full reductions are one launch (``mmp_reduce``) instead of a tree of
  launches plus a host read (``ndarray.py:1927-1951``);
* axis reductions run on the (outer, k, inner) view in place, without the
  transpose copy of ``ndarray._reduce_axis`` (``ndarray.py:2039-2047``);
* var/std are one pass (shifted moments), not mean -> broadcast subtract ->
  square -> mean (``ndarray.py:1823-1834``);
* a reduction of a lazy expression fuses the expression into the kernel;
* cumsum is a single-pass decoupled-look-back scan (``mmp_scan``).

Result dtypes are numpy's (the reference's CPU path): int32 sum -> int64,
int mean/var -> float64 (then ``resolve_dtype``), argmax -> int64, and
``argmax(axis=None)`` returns a Python ``int`` as the reference does
(``reductions.py:407``).
"""

from __future__ import annotations

import builtins
import ctypes
import math

import numpy as np

from . import _cuda_backend as _cb
from . import _fusion as _fu
from ._dtypes import MMP_CODES, resolve_dtype
from .ndarray import ndarray

__all__ = [
    "sum", "prod", "mean", "var", "std", "max", "min", "amax", "amin", "argmax", "argmin",
    "any", "all", "cumsum", "cumprod", "ptp", "diff", "average",
]

OPC = {
    "sum": 0, "prod": 1, "max": 2, "min": 3, "mean": 4, "var": 5, "std": 6, "argmax": 7,
    "argmin": 8, "nansum": 9, "nanmean": 10, "nanmax": 11, "nanmin": 12, "any": 13, "all": 14,
    "nanvar": 15, "nanstd": 16,
}

_NP_FN = {
    "sum": np.sum, "prod": np.prod, "max": np.max, "min": np.min, "mean": np.mean, "var": np.var,
    "std": np.std, "nansum": np.nansum, "nanmean": np.nanmean, "nanmax": np.nanmax,
    "nanmin": np.nanmin, "nanvar": np.nanvar, "nanstd": np.nanstd,
}

_NO_IDENTITY = {"max": "maximum", "min": "minimum", "argmax": "argmax", "argmin": "argmin",
                "nanmax": "fmax", "nanmin": "fmin"}

from ._config import get_config  # noqa: E402

_dt_cache: dict = {}
_CFG = get_config()


def _asarray(a) -> ndarray:
    if isinstance(a, ndarray):
        return a
    from .creation import asarray
    return asarray(a)


def out_dtype(kind: str, dt) -> np.dtype:
    """numpy's result dtype of reduction ``kind`` on ``dt``, resolved."""
    key = (kind, dt if isinstance(dt, np.dtype) else np.dtype(dt), _CFG.float64_behavior)
    r = _dt_cache.get(key)
    if r is None:
        if kind in ("argmax", "argmin"):
            r = np.dtype(np.int64)
        elif kind in ("any", "all"):
            r = np.dtype(np.bool_)
        else:
            r = resolve_dtype(np.asarray(_NP_FN[kind](np.ones(2, dtype=dt))).dtype)
        _dt_cache[key] = r
    return r


def _norm_axes(axis, ndim):
    if axis is None:
        return None
    ax = (axis,) if isinstance(axis, (int, np.integer)) else tuple(axis)
    out = []
    for a in ax:
        a = int(a)
        if not -ndim <= a < ndim:
            raise np.exceptions.AxisError(a, ndim)
        out.append(a % ndim)
    if len(set(out)) != len(out):
        raise ValueError("duplicate value in 'axis'")
    return tuple(sorted(out))


def _scalar_result(dt) -> ndarray:
    return ndarray._empty0(np.dtype(dt))


def _reduce(a, kind: str, axis=None, keepdims=False, ddof=0.0, dtype=None, out=None, partial=False,
            out_dt=None):
    # the common case first: a lazy expression reduced to one value
    if (axis is None and a.__class__ is ndarray and a._fusion_node is not None and dtype is None
            and not keepdims and not partial and out_dt is None):
        dt = a._dtype
        k = kind if (dt.kind == "f" or not kind.startswith("nan")) else kind[3:]
        if k not in _NO_IDENTITY or a.size:
            odt = _dt_cache.get((k, dt, _CFG.float64_behavior)) or out_dtype(k, dt)
            res = ndarray._empty0(odt)
            _fu.run_reduce(a._fusion_node, a._shape, OPC[k], res._buffer.ptr, odt, ddof)
            return res if out is None else _finish(res, out)
    if a.__class__ is not ndarray and a.__class__.__name__ == "DistArray":
        from . import distributed
        return distributed._reduce_call(a, kind, axis, keepdims, ddof, dtype, out)
    a = _asarray(a)
    if dtype is not None:
        a = a.astype(resolve_dtype(dtype), copy=False)
    if a._dtype.kind == "f" or kind not in ("nansum", "nanmean", "nanmax", "nanmin", "nanvar", "nanstd"):
        k = kind
    else:  # no NaN in integer/bool arrays (nan_ops.py:132-134)
        k = kind[3:]
    odt = out_dtype(k, a._dtype) if out_dt is None else np.dtype(out_dt)
    axes = _norm_axes(axis, a.ndim)
    if axes is not None and len(axes) == a.ndim:
        axes = None if not (k in ("argmax", "argmin") and a.ndim > 1) else axes
    if k in ("argmax", "argmin") and axes is not None and len(axes) > 1:
        raise TypeError("'tuple' object cannot be interpreted as an integer")
    opc = OPC[k]
    if axes is None:
        if a.size == 0 and k in _NO_IDENTITY:
            raise ValueError(f"zero-size array to reduction operation {_NO_IDENTITY[k]} which has no identity")
        res = _scalar_result(odt)
        part = None
        if a._fusion_node is not None:
            part = _fu.run_reduce(a._fusion_node, a._shape, opc, res._buffer.ptr, odt, ddof,
                                  want_partial=partial)
        else:
            src = a._ensure_contiguous()
            p = _cb.MmpPartial() if partial else None
            _cb.check(_cb.lib.mmp_reduce(opc, MMP_CODES[src._dtype], ctypes.c_void_p(src._ptr if src.size else 0),
                                         src.size, MMP_CODES[odt], ctypes.c_void_p(res._buffer.ptr),
                                         float(ddof), ctypes.byref(p) if p is not None else None),
                      f"{kind}")
            part = p
        if keepdims:
            res = res.reshape((1,) * a.ndim)
        if partial:
            return res, part
        return _finish(res, out)
    # ---- axis reduction on the (outer, k, inner) view
    shape = a._shape
    lo, hi = axes[0], axes[-1]
    adjacent = list(axes) == list(range(lo, hi + 1))
    if not adjacent:
        rest = [i for i in range(a.ndim) if i not in axes]
        a = a.transpose(rest + list(axes))._ensure_contiguous()
        shp2 = a._shape
        nr = len(rest)
        outer, kk, inner = math.prod(shp2[:nr]), math.prod(shp2[nr:]), 1
    else:
        outer, kk, inner = math.prod(shape[:lo]), math.prod(shape[lo:hi + 1]), math.prod(shape[hi + 1:])
    oshape = tuple(s for i, s in enumerate(shape) if i not in axes)
    if kk == 0:
        if k in _NO_IDENTITY:
            raise ValueError(f"zero-size array to reduction operation {_NO_IDENTITY[k]} which has no identity")
    res = ndarray._empty(oshape, odt)
    if res.size:
        if kk == 0:
            from . import creation
            fill = {"sum": 0, "nansum": 0, "prod": 1, "any": False, "all": True}.get(k, np.nan)
            res = creation.full(oshape, fill, dtype=odt)
        elif a._fusion_node is not None and adjacent:
            _fu.run_reduce(a._fusion_node, a._shape, opc, res._buffer.ptr, odt, ddof,
                           axis_split=(outer, kk, inner))
        else:
            src = a._ensure_contiguous()
            _cb.check(_cb.lib.mmp_reduce_axis(opc, MMP_CODES[src._dtype], ctypes.c_void_p(src._ptr), outer, kk,
                                              inner, MMP_CODES[odt], ctypes.c_void_p(res._buffer.ptr),
                                              float(ddof)), f"{kind}(axis)")
    if keepdims:
        kshape = tuple(1 if i in axes else s for i, s in enumerate(shape))
        res = res.reshape(kshape)
    return _finish(res, out)


def _finish(res: ndarray, out):
    if out is None:
        return res
    out[...] = res
    return out


def sum(a, axis=None, dtype=None, out=None, keepdims=False, initial=np._NoValue, where=np._NoValue):
    """Sum of array elements (int sums accumulate in 64 bits)."""
    if where is not np._NoValue:
        a = _asarray(a)
        from . import math_ops
        a = math_ops.where(where, a, 0)
    r = _reduce(a, "sum", axis, keepdims, dtype=dtype)
    if initial is not np._NoValue:
        r = r + initial
    return _finish(r, out)


def prod(a, axis=None, dtype=None, out=None, keepdims=False, initial=np._NoValue, where=np._NoValue):
    """Product of array elements."""
    r = _reduce(a, "prod", axis, keepdims, dtype=dtype)
    if initial is not np._NoValue:
        r = r * initial
    return _finish(r, out)


def mean(a, axis=None, dtype=None, out=None, keepdims=False, where=np._NoValue):
    """Arithmetic mean (computed in double, returned in numpy's dtype)."""
    return _reduce(a, "mean", axis, keepdims, dtype=dtype, out=out)


def var(a, axis=None, dtype=None, out=None, ddof=0, keepdims=False, where=np._NoValue, *, correction=None,
        mean=None):
    """Variance in one pass (shifted moments); ``correction`` aliases ddof."""
    if correction is not None:
        ddof = correction
    return _reduce(a, "var", axis, keepdims, ddof=float(ddof), dtype=dtype, out=out)


def std(a, axis=None, dtype=None, out=None, ddof=0, keepdims=False, where=np._NoValue, *, correction=None,
        mean=None):
    """Standard deviation in one pass; ``correction`` aliases ddof."""
    if correction is not None:
        ddof = correction
    return _reduce(a, "std", axis, keepdims, ddof=float(ddof), dtype=dtype, out=out)


def max(a, axis=None, out=None, keepdims=False, initial=np._NoValue, where=np._NoValue):
    """Maximum (NaN propagates)."""
    r = _reduce(a, "max", axis, keepdims)
    if initial is not np._NoValue:
        r = r._binary_op(initial, "max_op")
    return _finish(r, out)


def min(a, axis=None, out=None, keepdims=False, initial=np._NoValue, where=np._NoValue):
    """Minimum (NaN propagates)."""
    r = _reduce(a, "min", axis, keepdims)
    if initial is not np._NoValue:
        r = r._binary_op(initial, "min_op")
    return _finish(r, out)


amax = max
amin = min


def _arg(a, kind, axis, out, keepdims):
    if a.__class__.__name__ == "DistArray":
        from . import distributed
        return distributed._reduce_call(a, kind, axis, keepdims, 0.0, None, out)
    a = _asarray(a)
    if axis is None:
        if a.ndim == 0:
            return 0
        flat = a if a._fusion_node is not None else a._ensure_contiguous()
        if flat._fusion_node is not None:
            flat._materialize_if_lazy()
        r = _reduce(flat.reshape(-1), kind, None, False)
        if keepdims:
            r = r.reshape((1,) * a.ndim)
            return _finish(r, out)
        if out is not None:
            return _finish(r, out)
        return int(r.get())
    # axis arg-reductions return int32, as the reference's _reduce_axis
    # (reductions.py:410, ndarray.py:2015-2035) does on both of its paths
    return _reduce(a, kind, (int(axis),), keepdims, out=out, out_dt=np.int32)


def argmax(a, axis=None, out=None, keepdims=False):
    """Index of the maximum (first occurrence; the first NaN wins)."""
    return _arg(a, "argmax", axis, out, keepdims)


def argmin(a, axis=None, out=None, keepdims=False):
    """Index of the minimum (first occurrence; the first NaN wins)."""
    return _arg(a, "argmin", axis, out, keepdims)


def any(a, axis=None, out=None, keepdims=False, where=np._NoValue):
    """True if any element is non-zero."""
    return _reduce(a, "any", axis, keepdims, out=out)


def all(a, axis=None, out=None, keepdims=False, where=np._NoValue):
    """True if every element is non-zero."""
    return _reduce(a, "all", axis, keepdims, out=out)


# ---------------------------------------------------------------------------
# scans
# ---------------------------------------------------------------------------


def scan_out_dtype(dt) -> np.dtype:
    return np.dtype(np.cumsum(np.ones(1, dtype=dt)).dtype) if np.dtype(dt).kind != "f" else np.dtype(dt)


def _scan(a, op: int, axis=None, dtype=None, out=None, carry_ptr: int = 0):
    if a.__class__.__name__ == "DistArray":
        from . import distributed
        return distributed._scan_call(a, op, axis, dtype, out)
    a = _asarray(a)
    if dtype is not None:
        a = a.astype(resolve_dtype(dtype), copy=False)
    odt = scan_out_dtype(a._dtype)
    if axis is None:
        src = a.reshape(-1)._ensure_contiguous() if a._fusion_node is None else a._ensure_contiguous().reshape(-1)
        outer, kk, inner = 1, src.size, 1
        oshape = (src.size,)
    else:
        ax = _norm_axes(axis, a.ndim)[0]
        src = a._ensure_contiguous()
        shp = src._shape
        outer, kk, inner = math.prod(shp[:ax]), shp[ax], math.prod(shp[ax + 1:])
        oshape = shp
    res = ndarray._empty(oshape, odt)
    if res.size:
        _cb.check(_cb.lib.mmp_scan(op, MMP_CODES[src._dtype], ctypes.c_void_p(src._ptr), MMP_CODES[odt],
                                   ctypes.c_void_p(res._buffer.ptr), outer, kk, inner,
                                   ctypes.c_void_p(carry_ptr) if carry_ptr else None), "scan")
    return _finish(res, out)


def cumsum(a, axis=None, dtype=None, out=None):
    """Inclusive cumulative sum (int -> int64, as numpy)."""
    return _scan(a, 0, axis, dtype, out)


def cumprod(a, axis=None, dtype=None, out=None):
    """Inclusive cumulative product."""
    return _scan(a, 1, axis, dtype, out)


# ---------------------------------------------------------------------------
# range, differences, weighted mean (reductions.py:707-847 in the reference,
# which hands them to numpy below its size thresholds); here every one is
# device work built from the reductions and fused elementwise ops above.


def ptp(a, axis=None, out=None, keepdims=False):
    """max - min along ``axis`` (reductions.py:784-803): two device
    reductions and one fused subtract."""
    a = _asarray(a)
    return _finish(max(a, axis=axis, keepdims=keepdims) - min(a, axis=axis, keepdims=keepdims), out)


def diff(a, n=1, axis=-1, prepend=np._NoValue, append=np._NoValue):
    """n-th discrete difference along ``axis`` (reductions.py:707-781):
    ``a[1:] - a[:-1]`` on strided views, fused, n times; ``prepend`` /
    ``append`` are broadcast to one slab along ``axis`` and joined on the
    device first (numpy's rules)."""
    from .creation import asarray, empty

    a = _asarray(a)
    if n < 0:
        raise ValueError(f"order must be non-negative but got {n}")
    if a.ndim == 0:
        raise ValueError("diff requires input that is at least one dimensional")
    ax = axis % a.ndim
    if prepend is not np._NoValue or append is not np._NoValue:
        parts = []
        for extra, first in ((prepend, True), (append, False)):
            if extra is np._NoValue:
                continue
            e = asarray(extra)
            if e.ndim == 0:  # a scalar becomes a slab of length 1 along axis
                shp = list(a.shape)
                shp[ax] = 1
                e = e.reshape((1,) * a.ndim).broadcast_to(tuple(shp))
            parts.append((first, e))
        pre = [e for f, e in parts if f]
        post = [e for f, e in parts if not f]
        seq = pre + [a] + post
        dt = np.result_type(*[x.dtype for x in seq])
        tot = builtins.sum(x.shape[ax] for x in seq)
        shp = list(a.shape)
        shp[ax] = tot
        joined = empty(tuple(shp), dtype=dt)
        pos = 0
        for x in seq:
            idx = [slice(None)] * a.ndim
            idx[ax] = slice(pos, pos + x.shape[ax])
            joined[tuple(idx)] = x
            pos += x.shape[ax]
        a = joined
    hi = [slice(None)] * a.ndim
    lo = [slice(None)] * a.ndim
    hi[ax] = slice(1, None)
    lo[ax] = slice(None, -1)
    hi, lo = tuple(hi), tuple(lo)
    for _ in range(n):
        if a.dtype == np.bool_:
            a = a[hi] != a[lo]  # numpy: not_equal for booleans
        else:
            a = a[hi] - a[lo]
    return a


def average(a, axis=None, weights=None, returned=False, keepdims=False):
    """Weighted mean (reductions.py:823-846): ``sum(a * w) / sum(w)`` on the
    device, with 1-D weights laid along ``axis`` as numpy does; without
    weights, ``mean``.  ``returned`` also gives the sum of the weights."""
    from .creation import asarray, full

    a = _asarray(a)
    if weights is None:
        avg = mean(a, axis=axis, keepdims=keepdims)
        if returned:
            cnt = a.size if axis is None else math.prod(
                a.shape[i] for i in ((axis,) if isinstance(axis, int) else axis))
            return avg, full(avg.shape, cnt, dtype=avg.dtype)
        return avg
    w = asarray(weights)
    if w.shape != a.shape:
        if axis is None:
            raise TypeError("Axis must be specified when shapes of a and weights differ.")
        if w.ndim != 1:
            raise TypeError("1D weights expected when shapes of a and weights differ.")
        ax = axis % a.ndim
        if w.shape[0] != a.shape[ax]:
            raise ValueError("Length of weights not compatible with specified axis.")
        shp = [1] * a.ndim
        shp[ax] = w.shape[0]
        w = w.reshape(tuple(shp))
    rdt = np.result_type(a.dtype, w.dtype, np.float64 if a.dtype.kind in "iub" else a.dtype)
    rdt = resolve_dtype(rdt)
    aw = a.astype(rdt) * w.astype(rdt)
    wfull = w.astype(rdt) if w.shape == a.shape else w.astype(rdt).broadcast_to(a.shape)
    scl = sum(wfull, axis=axis, keepdims=keepdims)
    avg = sum(aw, axis=axis, keepdims=keepdims) / scl
    if returned:
        return avg, scl
    return avg
