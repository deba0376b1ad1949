"""Array creation (mirrors ``src/macmetalpy/creation.py``).

The reference builds CPU-resident arrays and uploads lazily on first GPU use
(``creation.py:36-114``, ``ndarray._ensure_gpu`` ``ndarray.py:352-368``);
here every array is created in device memory at once.  ``zeros``/``full``
fill on the device (memset or the fused fill kernel); host data is copied
with one H2D copy.
"""

from __future__ import annotations

import ctypes
import math
import numbers

import numpy as np

from . import _cuda_backend as _cb
from . import _fusion as _fu
from ._config import get_config
from ._dtypes import resolve_dtype
from .ndarray import ndarray

_CFG = get_config()

__all__ = [
    "array", "asarray", "asanyarray", "ascontiguousarray", "empty", "empty_like", "zeros", "zeros_like",
    "ones", "ones_like", "full", "full_like", "arange", "linspace", "asnumpy", "eye", "identity", "copy", "expand_dims",
]


def _shape(shape):
    if isinstance(shape, (numbers.Integral, np.integer)):
        return (int(shape),)
    return tuple(int(s) for s in shape)


def array(obj, dtype=None, copy=True, order="C", ndmin=0) -> ndarray:
    """Create a device array from ``obj`` (numpy array, list, scalar, ndarray).

    On a multi-rank job with ``set_config(shard_threshold=n)``, host data of
    at least n elements (and at least one dimension) becomes this rank's row
    block: a ``distributed.DistArray``."""
    if isinstance(obj, ndarray):
        r = obj.astype(dtype) if dtype is not None and np.dtype(dtype) != obj.dtype else (obj.copy() if copy else obj)
    else:
        if _CFG.shard_threshold is not None and obj.__class__.__name__ != "DistArray":
            from . import distributed
            d = distributed._shard_host(obj, dtype, _CFG.shard_threshold)
            if d is not None:
                return d
        host = np.asarray(obj, dtype=dtype)
        r = ndarray._from_numpy(host, resolve_dtype(dtype if dtype is not None else host.dtype))
    while r.ndim < ndmin:
        r = r.reshape((1,) + r.shape)
    return r


def asarray(obj, dtype=None, order=None) -> ndarray:
    """Like :func:`array` but returns ``obj`` itself when already suitable."""
    if isinstance(obj, ndarray) and (dtype is None or np.dtype(dtype) == obj.dtype):
        return obj
    if obj.__class__.__name__ == "DistArray" and dtype is None:
        return obj
    return array(obj, dtype=dtype, copy=False)


asanyarray = asarray


def ascontiguousarray(a, dtype=None) -> ndarray:
    return asarray(a, dtype)._ensure_contiguous()


def asnumpy(a, stream=None, order="C", out=None):
    """Device -> host (``cupy.asnumpy``)."""
    if isinstance(a, ndarray):
        return a.get(out=out)
    return np.asarray(a)


def empty(shape, dtype=None, order="C") -> ndarray:
    return ndarray._empty(_shape(shape), resolve_dtype(dtype))


def zeros(shape, dtype=None, order="C") -> ndarray:
    a = empty(shape, dtype)
    if a.nbytes:
        _cb.check(_cb.lib.mmp_memset(ctypes.c_void_p(a._buffer.ptr), 0, a.nbytes), "memset")
    return a


def full(shape, fill_value, dtype=None, order="C") -> ndarray:
    shape = _shape(shape)
    if dtype is None:
        dtype = np.asarray(fill_value).dtype if not isinstance(fill_value, float) else None
    dtype = resolve_dtype(dtype)
    a = ndarray._empty(shape, dtype)
    if a.size:
        v = np.asarray(fill_value).astype(dtype)
        if not v.any() and not (dtype.kind == "f" and np.signbit(v)):
            _cb.check(_cb.lib.mmp_memset(ctypes.c_void_p(a._buffer.ptr), 0, a.nbytes), "memset")
        else:
            _fu.run_elementwise(_fu.ScalarNode(v, dtype), a._buffer.ptr, shape)
    return a


def ones(shape, dtype=None, order="C") -> ndarray:
    return full(shape, 1, dtype if dtype is not None else resolve_dtype(None))


def empty_like(a, dtype=None, order="K", subok=True, shape=None) -> ndarray:
    return empty(a.shape if shape is None else shape, a.dtype if dtype is None else dtype)


def zeros_like(a, dtype=None, order="K", subok=True, shape=None) -> ndarray:
    return zeros(a.shape if shape is None else shape, a.dtype if dtype is None else dtype)


def ones_like(a, dtype=None, order="K", subok=True, shape=None) -> ndarray:
    return ones(a.shape if shape is None else shape, a.dtype if dtype is None else dtype)


def full_like(a, fill_value, dtype=None, order="K", subok=True, shape=None) -> ndarray:
    return full(a.shape if shape is None else shape, fill_value, a.dtype if dtype is None else dtype)


def arange(start, stop=None, step=1, dtype=None) -> ndarray:
    return ndarray._from_numpy(np.arange(start, stop, step, dtype=dtype) if stop is not None
                               else np.arange(start, dtype=dtype))


def linspace(start, stop, num=50, endpoint=True, retstep=False, dtype=None, axis=0):
    r = np.linspace(start, stop, num, endpoint=endpoint, retstep=retstep, dtype=dtype, axis=axis)
    if retstep:
        return ndarray._from_numpy(r[0]), r[1]
    return ndarray._from_numpy(r)


def eye(N, M=None, k=0, dtype=None) -> ndarray:
    return ndarray._from_numpy(np.eye(N, M, k, dtype=resolve_dtype(dtype)))


def identity(n, dtype=None) -> ndarray:
    return eye(n, dtype=dtype)


def copy(a, order="K") -> ndarray:
    """A device copy of ``a`` (math_ops copy in the reference)."""
    return asarray(a).copy()


def expand_dims(a, axis) -> ndarray:
    """View of ``a`` with length-1 axes inserted at ``axis`` (an int or a
    tuple, numpy's normalisation of negative positions)."""
    a = asarray(a)
    axes = (axis,) if isinstance(axis, int) else tuple(axis)
    nd = a.ndim + len(axes)
    norm = sorted(ax % nd if -nd <= ax < nd else _bad_axis(ax, nd) for ax in axes)
    if len(set(norm)) != len(norm):
        raise ValueError("repeated axis")
    for ax in norm:
        a = a.expand_dims(ax)
    return a


def _bad_axis(ax, nd):
    raise np.exceptions.AxisError(ax, nd)

