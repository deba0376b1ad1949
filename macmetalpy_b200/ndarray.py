"""Device-resident N-dimensional array for the B200 backend.

Mirrors ``class ndarray`` of the reference (``src/macmetalpy/ndarray.py:236``):
the same attribute set -- ``_buffer``, ``_shape``, ``_dtype``, ``_strides``
(element strides), ``_offset`` (elements), ``_base``, ``_fusion_node`` -- and
the same public surface for the hot path (operators, ``get``/``set``, views,
reductions, ``cumsum``, ``@``).  What differs, by design:

* there is no CPU residency and no size-threshold router
  (``ndarray.py:40-132``): every array lives in device memory and every op
  runs on the GPU (no CPU fallback, float64 included);
* every fuseable elementwise op is lazy (the reference makes unary ops lazy
  always and binary ops lazy when an operand is lazy,
  ``ndarray.py:1071-1103,1204-1235``); the graph is evaluated by one
  generated kernel at a materialisation point, and a reduction of a lazy
  array fuses the expression into the reduction;
* broadcasting and strided operands are indexed in the kernel, never
  copied;
* result dtypes follow numpy's ufunc type resolution followed by
  ``resolve_dtype`` (so int32 sums are int64, argmax indices int64, as on
  the reference's CPU path).
"""

from __future__ import annotations

import ctypes
import math
import numbers
from typing import Optional, Tuple

import numpy as np

from . import _cuda_backend as _cb
from . import _fusion as _fu
from ._broadcasting import broadcast_shapes
from ._dtypes import MMP_CODES, resolve_dtype

__all__ = ["ndarray"]

_STRIDE_CACHE: dict = {}


def _c_contiguous_strides(shape) -> Tuple[int, ...]:
    s = _STRIDE_CACHE.get(shape)
    if s is not None:
        return s
    st = [1] * len(shape)
    for i in range(len(shape) - 2, -1, -1):
        st[i] = st[i + 1] * shape[i + 1]
    r = tuple(st)
    if len(_STRIDE_CACHE) < 1024:
        _STRIDE_CACHE[shape] = r
    return r


# ---------------------------------------------------------------------------
# dtype resolution of elementwise ops (numpy ufunc rules + resolve_dtype)
# ---------------------------------------------------------------------------

from ._config import get_config  # noqa: E402

_CFG = get_config()

_RES_CACHE: dict = {}
_STRIDES_CACHE: dict = {}


def _operand_spec(x):
    """dtype key for numpy's resolver: arrays/np scalars by dtype, Python
    scalars as weak types (NEP 50)."""
    if isinstance(x, ndarray):
        return x._dtype
    if isinstance(x, (bool, np.bool_)) and not isinstance(x, np.generic):
        return np.dtype(np.bool_)  # a Python bool is not a weak scalar (NEP 50)
    if isinstance(x, np.generic):
        return x.dtype
    if isinstance(x, numbers.Integral):
        return int
    if isinstance(x, numbers.Real):
        return float
    if isinstance(x, numbers.Complex):
        raise TypeError("complex scalars are not supported on the device path")
    return np.asarray(x).dtype


def _resolve(op_name: str, specs: tuple):
    """(loop_dtype, out_dtype) for an elementwise op after resolve_dtype."""
    cfg = _CFG
    key = (op_name, specs, cfg.float64_behavior, cfg.default_float_dtype)
    r = _RES_CACHE.get(key)
    if r is not None:
        return r
    uf = _fu._UNARY_UFUNC.get(op_name) or _fu._BINARY_UFUNC[op_name]
    dts = uf.resolve_dtypes(tuple(specs) + (None,))
    loop = resolve_dtype(dts[0])
    out = resolve_dtype(dts[-1])
    r = (loop, out)
    _RES_CACHE[key] = r
    return r


_SCALAR_TYPES = (bool, int, float)


def _elementwise_fast(op_name, operands):
    """The common case of ``ndarray._elementwise`` in one pass, or None.

    Taken when every operand is an ndarray or a Python / numpy scalar, the
    array operands share one shape, no operand needs a cast to the loop
    dtype, and no operand graph reaches the depth cap; anything else goes
    the general way (same result, more checks)."""
    if len(operands) == 1:  # unary on an array: no lists
        o = operands[0]
        if o.__class__ is not ndarray:
            return None
        loop, out = _resolve(op_name, (o._dtype,))
        nd = o._fusion_node
        if nd is None:
            nd = _fu.InputNode(o)
        elif nd._depth >= _fu._MAX_DEPTH:
            return None
        if nd._dtype != loop:
            return None
        return ndarray._lazy(_fu.unary_node(op_name, nd, o._shape, out, loop))
    specs = []
    shape = None
    for o in operands:
        if o.__class__ is ndarray:
            if shape is None:
                shape = o._shape
            elif o._shape != shape:
                return None
            specs.append(o._dtype)
        elif o.__class__ in _SCALAR_TYPES:
            specs.append(np.dtype(np.bool_) if o.__class__ is bool else o.__class__)
        elif isinstance(o, np.generic):
            specs.append(o.dtype)
        else:
            return None
    if shape is None:
        return None
    loop, out = _resolve(op_name, tuple(specs))
    nodes = []
    for o in operands:
        if o.__class__ is ndarray:
            nd = o._fusion_node
            if nd is None:
                nd = _fu.InputNode(o)
            elif nd._depth + 1 > _fu._MAX_DEPTH:
                return None
            if nd._dtype != loop:
                return None
        else:
            nd = _fu.ScalarNode(o, loop)
        nodes.append(nd)
    if len(nodes) == 1:
        node = _fu.unary_node(op_name, nodes[0], shape, out, loop)
    else:
        node = _fu.binary_node(op_name, nodes[0], nodes[1], shape, out, loop)
    return ndarray._lazy(node)


class ndarray:
    """CuPy-style GPU array on B200.  Construct through
    :mod:`macmetalpy_b200.creation` functions."""

    __array_priority__ = 100.0
    _fusion_node = None

    def __init__(self, buffer, shape, dtype, strides: Optional[tuple] = None, offset: int = 0,
                 base: Optional["ndarray"] = None) -> None:
        self._buffer = buffer
        self._shape = tuple(int(s) for s in shape)
        self._dtype = np.dtype(dtype)
        self._strides = tuple(strides) if strides is not None else _c_contiguous_strides(self._shape)
        self._offset = int(offset)
        self._base = base
        self._fusion_node = None

    # ------------------------------------------------------------------ construction
    @classmethod
    def _from_buffer(cls, buffer, shape, dtype, strides=None, offset=0, base=None) -> "ndarray":
        return cls(buffer, shape, dtype, strides=strides, offset=offset, base=base)

    @classmethod
    def _empty(cls, shape, dtype) -> "ndarray":
        shape = tuple(int(s) for s in shape)
        dtype = np.dtype(dtype)
        n = math.prod(shape) if shape else 1
        buf = _cb.DeviceBuffer(max(n * dtype.itemsize, 1))
        return cls(buf, shape, dtype)

    @classmethod
    def _empty0(cls, dtype) -> "ndarray":
        """A new 0-d array of ``dtype`` (an np.dtype), uninitialised."""
        a = cls.__new__(cls)
        a._buffer = _cb.DeviceBuffer(dtype.itemsize)
        a._shape = ()
        a._dtype = dtype
        a._strides = ()
        a._offset = 0
        a._base = None
        a._fusion_node = None
        return a

    @classmethod
    def _lazy(cls, node) -> "ndarray":
        a = cls.__new__(cls)
        a._buffer = None
        a._shape = shp = tuple(node._shape)
        a._dtype = node._dtype
        st = _STRIDES_CACHE.get(shp)
        if st is None:
            if len(_STRIDES_CACHE) > 4096:
                _STRIDES_CACHE.clear()
            st = _STRIDES_CACHE[shp] = _c_contiguous_strides(shp)
        a._strides = st
        a._offset = 0
        a._base = None
        a._fusion_node = node
        return a

    @classmethod
    def _from_numpy(cls, arr: np.ndarray, dtype=None) -> "ndarray":
        """Upload a host array (after dtype resolution) into a new buffer."""
        arr = np.asarray(arr)
        target = resolve_dtype(dtype if dtype is not None else arr.dtype)
        host = np.asarray(arr, dtype=target, order="C")  # keeps 0-d shapes (ascontiguousarray makes them 1-d)
        out = cls._empty(host.shape, target)
        if host.nbytes:
            _cb.check(_cb.lib.mmp_h2d(ctypes.c_void_p(out._buffer.ptr), host.ctypes.data_as(ctypes.c_void_p),
                                      host.nbytes), "h2d")
        return out

    # ------------------------------------------------------------------ properties
    @property
    def shape(self) -> Tuple[int, ...]:
        return self._shape

    @shape.setter
    def shape(self, value):
        r = self.reshape(value)
        self._materialize_if_lazy()
        self._shape, self._strides, self._offset, self._buffer = r._shape, r._strides, r._offset, r._buffer

    @property
    def dtype(self) -> np.dtype:
        return self._dtype

    @property
    def ndim(self) -> int:
        return len(self._shape)

    @property
    def size(self) -> int:
        return math.prod(self._shape) if self._shape else 1

    @property
    def itemsize(self) -> int:
        return self._dtype.itemsize

    @property
    def nbytes(self) -> int:
        return self.size * self.itemsize

    @property
    def strides(self) -> Tuple[int, ...]:
        """Byte strides (element strides * itemsize), as CuPy reports them."""
        return tuple(s * self.itemsize for s in self._strides)

    @property
    def T(self) -> "ndarray":
        return self.transpose()

    @property
    def base(self):
        return self._base

    @property
    def device(self):
        return f"cuda:{_cb.CudaBackend().device}"

    @property
    def real(self) -> "ndarray":
        return self

    @property
    def _ptr(self) -> int:
        """Device address of element [0, ..., 0]."""
        if self._fusion_node is not None:
            self._materialize_if_lazy()
        return self._buffer.ptr + self._offset * self._dtype.itemsize

    @property
    def data_ptr(self) -> int:
        return self._ptr

    @property
    def __cuda_array_interface__(self):
        self._materialize_if_lazy()
        return {
            "shape": self._shape,
            "typestr": self._dtype.str,
            "data": (self._ptr, False),
            "strides": None if self._is_c_contiguous() else self.strides,
            "version": 3,
            "stream": _cb.CudaBackend().stream_ptr() or None,
        }

    # ------------------------------------------------------------------ laziness / layout
    def _materialize_if_lazy(self) -> None:
        if self._fusion_node is not None:
            _fu.materialize(self)

    def _is_c_contiguous(self) -> bool:
        if self._fusion_node is not None:
            return True
        if self.size <= 1:
            return True
        exp = _c_contiguous_strides(self._shape)
        return all(s == e for s, e, d in zip(self._strides, exp, self._shape) if d != 1)

    def _node(self):
        """Fusion node standing for this array's value."""
        if self._fusion_node is not None:
            return self._fusion_node
        return _fu.InputNode(self)

    def _ensure_contiguous(self) -> "ndarray":
        """Return self if C-contiguous (materialising a lazy graph), else a
        contiguous copy made by the fused copy kernel."""
        if self._fusion_node is not None:
            self._materialize_if_lazy()
            return self
        if self._is_c_contiguous():
            return self
        return self._contiguous_copy()

    def _contiguous_copy(self) -> "ndarray":
        out = ndarray._empty(self._shape, self._dtype)
        _fu.run_elementwise(_fu.InputNode(self), out._buffer.ptr, self._shape)
        return out

    # ------------------------------------------------------------------ host transfer
    def get(self, stream=None, order="C", out=None) -> np.ndarray:
        """Copy to host and return a numpy array.  Without ``stream`` it
        synchronises; with a side stream (``macmetalpy_b200.cuda.Stream``)
        the copy waits for the kernels enqueued so far and runs
        asynchronously -- synchronise the stream before reading ``out``."""
        a = self._ensure_contiguous()
        host = np.empty(self._shape, dtype=self._dtype) if out is None else out
        if out is not None and (out.shape != self._shape or out.dtype != self._dtype
                                or not out.flags.c_contiguous):
            raise ValueError("out must be a C-contiguous host array of this shape and dtype")
        if host.nbytes:
            if stream is None or getattr(stream, "ptr", None) is None:
                _cb.check(_cb.lib.mmp_d2h(host.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(a._ptr),
                                          host.nbytes), "d2h")
            else:
                from .cuda import Event
                stream.wait_event(Event().record(None))
                _cb.check(_cb.lib.mmp_d2h_async(host.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(a._ptr),
                                                host.nbytes, ctypes.c_void_p(stream.ptr)), "d2h_async")
        return host

    def set(self, arr, stream=None) -> None:
        """Copy host data into this array (broadcast to its shape).  With a
        side stream the copy runs on it, asynchronously, and later kernels
        wait for it; ``arr`` must then be an unchanged, C-contiguous array of
        this shape and dtype (pinned for a copy that does not block)."""
        self._materialize_if_lazy()
        if stream is not None and getattr(stream, "ptr", None) is not None and self._is_c_contiguous():
            host = arr
            if not (isinstance(host, np.ndarray) and host.shape == self._shape and host.dtype == self._dtype
                    and host.flags.c_contiguous):
                raise ValueError("set(stream=...) needs a C-contiguous host array of this shape and dtype")
            if host.nbytes:
                from .cuda import Event
                _cb.check(_cb.lib.mmp_h2d_async(ctypes.c_void_p(self._ptr), host.ctypes.data_as(ctypes.c_void_p),
                                                host.nbytes, ctypes.c_void_p(stream.ptr)), "h2d_async")
                ev = Event().record(stream)
                _cb.check(_cb.lib.mmp_stream_wait_event(None, ctypes.c_void_p(ev.ptr)), "stream wait")
            return
        host = np.asarray(np.broadcast_to(np.asarray(arr, dtype=self._dtype), self._shape), order="C")
        if self._is_c_contiguous():
            if host.nbytes:
                _cb.check(_cb.lib.mmp_h2d(ctypes.c_void_p(self._ptr), host.ctypes.data_as(ctypes.c_void_p),
                                          host.nbytes), "h2d")
            return
        tmp = ndarray._from_numpy(host, self._dtype)
        _fu.run_elementwise(_fu.InputNode(tmp), self._ptr, self._shape, out_strides=self._strides)

    def __array__(self, dtype=None, copy=None):
        a = self.get()
        return a.astype(dtype) if dtype is not None else a

    def tolist(self):
        return self.get().tolist()

    def item(self, *args):
        return self.get().item(*args)

    # Python scalar conversions: size-1 arrays only, with the reference's
    # messages (ndarray.py:2464-2495)
    def _one(self):
        if self.size != 1:
            raise TypeError("only size-1 arrays can be converted to Python scalars")
        return self.get().reshape(-1)[0]

    def __float__(self):
        return float(self._one())

    def __int__(self):
        return int(self._one())

    def __complex__(self):
        return complex(self._one())

    def __index__(self):
        if self._dtype.kind not in "iub":
            raise TypeError("only integer arrays can be used as an index")
        return int(self._one())

    def __bool__(self):
        if self.size != 1:
            raise ValueError("The truth value of an array with more than one element is ambiguous.")
        return bool(self.get())

    def __len__(self):
        if not self._shape:
            raise TypeError("len() of unsized object")
        return self._shape[0]

    def __iter__(self):
        if not self._shape:
            raise TypeError("iteration over a 0-d array")
        for i in range(self._shape[0]):
            yield self[i]

    def __repr__(self):
        return "array(" + np.array2string(self.get(), separator=", ", prefix="array(") + \
            (f", dtype={self._dtype})" if self._dtype not in (np.float32, np.int64, np.bool_) else ")")

    def __str__(self):
        return str(self.get())

    def __format__(self, spec):
        if self.ndim == 0:
            return format(self.get()[()], spec)
        return str(self)

    # ------------------------------------------------------------------ views
    def _view(self, shape, strides, offset) -> "ndarray":
        self._materialize_if_lazy()
        return ndarray._from_buffer(self._buffer, shape, self._dtype, strides=strides, offset=offset,
                                    base=self._base if self._base is not None else self)

    def reshape(self, *new_shape, order="C") -> "ndarray":
        if len(new_shape) == 1 and isinstance(new_shape[0], (tuple, list)):
            new_shape = tuple(new_shape[0])
        new_shape = tuple(int(s) for s in new_shape)
        if new_shape.count(-1) > 1:
            raise ValueError("can only specify one unknown dimension")
        if -1 in new_shape:
            known = math.prod(s for s in new_shape if s != -1)
            if known == 0 or self.size % known != 0:
                raise ValueError(f"cannot reshape array of size {self.size} into shape {new_shape}")
            new_shape = tuple(self.size // known if s == -1 else s for s in new_shape)
        if math.prod(new_shape) != self.size:
            raise ValueError(f"cannot reshape array of size {self.size} into shape {new_shape}")
        if self._fusion_node is not None:
            self._materialize_if_lazy()
        a = self if self._is_c_contiguous() else self._contiguous_copy()
        return a._view(new_shape, _c_contiguous_strides(new_shape), a._offset)

    def transpose(self, *axes) -> "ndarray":
        if len(axes) == 1 and (axes[0] is None or isinstance(axes[0], (tuple, list))):
            axes = axes[0]
        if not axes:
            axes = tuple(reversed(range(self.ndim)))
        axes = tuple(a % self.ndim for a in axes) if self.ndim else ()
        if sorted(axes) != list(range(self.ndim)):
            raise ValueError("axes don't match array")
        self._materialize_if_lazy()
        return self._view(tuple(self._shape[a] for a in axes), tuple(self._strides[a] for a in axes),
                          self._offset)

    def swapaxes(self, a1, a2) -> "ndarray":
        ax = list(range(self.ndim))
        ax[a1], ax[a2] = ax[a2], ax[a1]
        return self.transpose(ax)

    def ravel(self, order="C") -> "ndarray":
        return self.reshape(-1)

    def flatten(self, order="C") -> "ndarray":
        return self.copy().reshape(-1)

    def squeeze(self, axis=None) -> "ndarray":
        self._materialize_if_lazy()
        if axis is None:
            keep = [i for i, s in enumerate(self._shape) if s != 1]
        else:
            ax = (axis,) if isinstance(axis, int) else tuple(axis)
            ax = tuple(a % self.ndim for a in ax)
            for a in ax:
                if self._shape[a] != 1:
                    raise ValueError("cannot select an axis to squeeze out which has size not equal to one")
            keep = [i for i in range(self.ndim) if i not in ax]
        return self._view(tuple(self._shape[i] for i in keep), tuple(self._strides[i] for i in keep),
                          self._offset)

    def expand_dims(self, axis) -> "ndarray":
        self._materialize_if_lazy()
        nd = self.ndim + 1
        axis = axis % nd
        shp = list(self._shape)
        st = list(self._strides)
        shp.insert(axis, 1)
        st.insert(axis, 0)
        return self._view(tuple(shp), tuple(st), self._offset)

    def broadcast_to(self, shape) -> "ndarray":
        self._materialize_if_lazy()
        shape = tuple(shape)
        bs = broadcast_shapes(self._shape, shape)
        if bs != shape:
            raise ValueError(f"cannot broadcast {self._shape} to {shape}")
        st = _fu._bcast_strides(self._shape, self._strides, shape)
        return self._view(shape, tuple(st), self._offset)

    def _basic_index(self, key):
        """(shape, strides, offset) for a basic index key, or None."""
        if not isinstance(key, tuple):
            key = (key,)
        for k in key:
            if isinstance(k, (bool, np.bool_)) or not isinstance(k, (numbers.Integral, slice, type(None),
                                                                     type(Ellipsis))):
                return None
        if sum(1 for k in key if k is Ellipsis) > 1:
            raise IndexError("an index can only have a single ellipsis ('...')")
        n_idx = sum(1 for k in key if k is not None and k is not Ellipsis)
        if n_idx > self.ndim:
            raise IndexError(f"too many indices for array: array is {self.ndim}-dimensional, "
                             f"but {n_idx} were indexed")
        if Ellipsis in key:
            i = key.index(Ellipsis)
            key = key[:i] + (slice(None),) * (self.ndim - n_idx) + key[i + 1:]
        shp, st = [], []
        off = self._offset
        dim = 0
        for k in key:
            if k is None:
                shp.append(1)
                st.append(0)
            elif isinstance(k, numbers.Integral):
                size = self._shape[dim]
                i = int(k)
                if i < 0:
                    i += size
                if not 0 <= i < size:
                    raise IndexError(f"index {k} is out of bounds for axis {dim} with size {size}")
                off += i * self._strides[dim]
                dim += 1
            else:
                size = self._shape[dim]
                start, stop, step = k.indices(size)
                length = len(range(start, stop, step))
                off += start * self._strides[dim] if length else 0
                shp.append(length)
                st.append(self._strides[dim] * step)
                dim += 1
        while dim < self.ndim:
            shp.append(self._shape[dim])
            st.append(self._strides[dim])
            dim += 1
        return tuple(shp), tuple(st), off

    def __getitem__(self, key):
        self._materialize_if_lazy()
        r = self._basic_index(key)
        if r is not None:
            return self._view(*r)
        # advanced (integer / boolean array) indexing: device gather
        from . import _advindex
        return _advindex.getitem(self, key)

    def __setitem__(self, key, value):
        self._materialize_if_lazy()
        r = self._basic_index(key)
        if r is None:
            # advanced indexing: device scatter (or a fused select for a mask)
            from . import _advindex
            _advindex.setitem(self, key, value)
            return
        shp, st, off = r
        target = self._view(shp, st, off)
        if target.size == 0:
            return
        if isinstance(value, ndarray):
            node = value._node()
            if value._dtype != self._dtype:
                node = _fu.CastNode(node, self._dtype)
        elif isinstance(value, (numbers.Number, np.generic)):
            node = _fu.ScalarNode(value, self._dtype)
        else:
            v = ndarray._from_numpy(np.asarray(value), self._dtype)
            node = v._node()
        if broadcast_shapes(node._shape, shp) != shp:
            raise ValueError(f"could not broadcast input array from shape {node._shape} into shape {shp}")
        _fu.run_elementwise(node, target._ptr, shp, out_strides=st)

    # ------------------------------------------------------------------ copies / casts
    def copy(self, order="C") -> "ndarray":
        if self._fusion_node is not None:
            self._materialize_if_lazy()
        out = ndarray._empty(self._shape, self._dtype)
        if self.size:
            if self._is_c_contiguous():
                _cb.check(_cb.lib.mmp_d2d(ctypes.c_void_p(out._buffer.ptr), ctypes.c_void_p(self._ptr),
                                          self.nbytes), "d2d")
            else:
                _fu.run_elementwise(_fu.InputNode(self), out._buffer.ptr, self._shape)
        return out

    def astype(self, dtype, copy=True) -> "ndarray":
        dtype = resolve_dtype(dtype)
        if dtype == self._dtype and not copy:
            return self
        if dtype == self._dtype:
            return self.copy()
        return ndarray._lazy(_fu.CastNode(self._node(), dtype))

    def fill(self, value) -> None:
        self[...] = value

    def view(self, dtype=None):
        if dtype is None:
            return self._view(self._shape, self._strides, self._offset)
        dtype = np.dtype(dtype)
        if dtype.itemsize != self._dtype.itemsize:
            raise ValueError("view with a different itemsize is not supported")
        a = self._ensure_contiguous()
        return ndarray._from_buffer(a._buffer, a._shape, dtype, a._strides, a._offset, a)

    # ------------------------------------------------------------------ elementwise core
    @staticmethod
    def _to_node(x, target_dtype, shape_hint=None):
        """Node for operand ``x`` cast to ``target_dtype``."""
        if isinstance(x, ndarray):
            node = x._fusion_node if x._fusion_node is not None else _fu.InputNode(x)
        elif isinstance(x, (numbers.Number, np.generic)):
            return _fu.ScalarNode(x, target_dtype)
        else:
            node = ndarray._from_numpy(np.asarray(x))._node()
        if node._dtype != target_dtype:
            node = _fu.CastNode(node, target_dtype)
        return node

    @staticmethod
    def _elementwise(op_name: str, *operands) -> "ndarray":
        # fast path: every operand an ndarray or a Python / numpy scalar, the
        # array operands of one shape, no cast and no depth flush needed
        fast = _elementwise_fast(op_name, operands)
        if fast is not None:
            return fast
        for o in operands:
            if o.__class__.__name__ == "DistArray":  # block-distributed: the op on this rank's blocks
                from . import distributed
                return distributed._ufunc(op_name, operands)
        ops = []
        specs = []
        shape = None
        same = True
        for o in operands:
            if isinstance(o, ndarray):
                specs.append(o._dtype)
            elif isinstance(o, (numbers.Number, np.generic)):
                specs.append(_operand_spec(o))
            else:
                o = ndarray._from_numpy(np.asarray(o))
                specs.append(o._dtype)
            if isinstance(o, ndarray):
                if shape is None:
                    shape = o._shape
                elif o._shape != shape:
                    same = False
            ops.append(o)
        loop, out = _resolve(op_name, tuple(specs))
        if shape is None:
            shape = ()
        elif not same:
            shape = broadcast_shapes(*[o._shape if isinstance(o, ndarray) else () for o in ops])
        nodes = [ndarray._to_node(o, loop) for o in ops]
        # flush operands whose graphs would exceed the reference's depth cap
        for i, (o, nd) in enumerate(zip(ops, nodes)):
            if nd._depth + 1 > _fu._MAX_DEPTH and isinstance(o, ndarray) and o._fusion_node is not None:
                o._materialize_if_lazy()
                nodes[i] = ndarray._to_node(o, loop)
        if len(nodes) == 1:
            node = _fu.UnaryOpNode(op_name, nodes[0], shape, out, in_dtype=loop)
        else:
            node = _fu.BinaryOpNode(op_name, nodes[0], nodes[1], shape, out, in_dtype=loop)
        return ndarray._lazy(node)

    @staticmethod
    def _select(cond: "ndarray", x, y) -> "ndarray":
        """Lazy ``where(cond, x, y)`` with numpy's result dtype."""
        ops = [o if isinstance(o, (ndarray, numbers.Number, np.generic)) else ndarray._from_numpy(np.asarray(o))
               for o in (x, y)]
        specs = [o._dtype if isinstance(o, ndarray) else _operand_spec(o) for o in ops]
        dt = resolve_dtype(np.result_type(*[s if isinstance(s, np.dtype) else s(0) for s in specs]))
        shape = broadcast_shapes(cond._shape, *[o._shape if isinstance(o, ndarray) else () for o in ops])
        node = _fu.SelectNode(cond._node(), ndarray._to_node(ops[0], dt), ndarray._to_node(ops[1], dt), shape, dt)
        return ndarray._lazy(node)

    def _unary_op(self, op_name: str) -> "ndarray":
        r = _elementwise_fast(op_name, (self,))
        return r if r is not None else ndarray._elementwise(op_name, self)

    def _binary_op(self, other, op_name: str) -> "ndarray":
        if op_name == "pow_op" and other.__class__ is not ndarray and self._dtype.kind == "f" \
                and (other.__class__ in _SCALAR_TYPES or isinstance(other, (numbers.Number, np.generic))
                     or np.ndim(other) == 0):
            e = float(other)
            if e == 2.0:  # numpy's fast scalar power: x**2 is square(x)
                return self._unary_op("square_op")
        r = _elementwise_fast(op_name, (self, other))
        return r if r is not None else ndarray._elementwise(op_name, self, other)

    def _rbinary_op(self, other, op_name: str) -> "ndarray":
        return ndarray._elementwise(op_name, other, self)

    # arithmetic
    def __add__(self, o): return self._binary_op(o, "add_op")
    def __radd__(self, o): return self._rbinary_op(o, "add_op")
    def __sub__(self, o): return self._binary_op(o, "sub_op")
    def __rsub__(self, o): return self._rbinary_op(o, "sub_op")
    def __mul__(self, o): return self._binary_op(o, "mul_op")
    def __rmul__(self, o): return self._rbinary_op(o, "mul_op")
    def __truediv__(self, o): return self._binary_op(o, "div_op")
    def __rtruediv__(self, o): return self._rbinary_op(o, "div_op")
    # `//` and `%` cast a non-array operand to this array's dtype first, as the
    # reference does (creation.array(np.asarray(other), dtype=self._dtype),
    # ndarray.py:2501-2530)
    def _own(self, o):
        return o if isinstance(o, ndarray) else np.asarray(o).astype(self._dtype)[()]

    def __floordiv__(self, o): return self._binary_op(self._own(o), "floor_divide_op")
    def __rfloordiv__(self, o): return self._rbinary_op(self._own(o), "floor_divide_op")
    def __mod__(self, o): return self._binary_op(self._own(o), "mod_op")
    def __rmod__(self, o): return self._rbinary_op(self._own(o), "mod_op")
    def __pow__(self, o): return self._binary_op(o, "pow_op")
    def __rpow__(self, o): return self._rbinary_op(o, "pow_op")
    def __neg__(self): return self._unary_op("neg_op")
    def __pos__(self): return self._unary_op("positive_op")
    def __abs__(self): return self._unary_op("abs_op")

    def __divmod__(self, o):
        return self.__floordiv__(o), self.__mod__(o)

    # comparisons
    def __lt__(self, o): return self._binary_op(o, "lt_op")
    def __le__(self, o): return self._binary_op(o, "le_op")
    def __gt__(self, o): return self._binary_op(o, "gt_op")
    def __ge__(self, o): return self._binary_op(o, "ge_op")
    def __eq__(self, o): return self._binary_op(o, "eq_op")
    def __ne__(self, o): return self._binary_op(o, "ne_op")
    __hash__ = None

    # in-place: evaluate into this array's own memory
    def _inplace(self, o, op_name):
        r = self._binary_op(o, op_name)
        node = r._fusion_node
        if node._dtype != self._dtype:
            node = _fu.CastNode(node, self._dtype)
        self._materialize_if_lazy()
        _fu.run_elementwise(node, self._ptr, self._shape, out_strides=self._strides)
        return self

    def _inplace_result(self, r):
        """Write the (lazy) result ``r`` into this array, cast to its dtype."""
        node = r._node()
        if node._dtype != self._dtype:
            node = _fu.CastNode(node, self._dtype)
        self._materialize_if_lazy()
        _fu.run_elementwise(node, self._ptr, self._shape, out_strides=self._strides)
        return self

    # boolean / bitwise operators, dispatched as the reference does
    # (ndarray.py:1670-1700, 2549-2645): on integer arrays &, |, ^, ~ are the
    # int32 bitwise ops of bitwise_ops; on bool and float arrays &, |, ^ are
    # numpy's logical ops (the other operand taken as bool) and ~ is logical
    # not (of the int32 cast, for floats); << and >> are always the int32
    # shifts.  In-place forms cast the result back to this array's dtype.
    def _logic_bits(self, o, bits, logic, rev=False):
        from . import bitwise_ops, logic_ops
        if self._dtype.kind in "iu":
            f = getattr(bitwise_ops, bits)
        else:
            f = getattr(logic_ops, logic)
            if not isinstance(o, ndarray):
                o = np.asarray(o).astype(np.bool_)[()]
        return f(o, self) if rev else f(self, o)

    def __and__(self, o): return self._logic_bits(o, "bitwise_and", "logical_and")
    def __rand__(self, o): return self._logic_bits(o, "bitwise_and", "logical_and", True)
    def __or__(self, o): return self._logic_bits(o, "bitwise_or", "logical_or")
    def __ror__(self, o): return self._logic_bits(o, "bitwise_or", "logical_or", True)
    def __xor__(self, o): return self._logic_bits(o, "bitwise_xor", "logical_xor")
    def __rxor__(self, o): return self._logic_bits(o, "bitwise_xor", "logical_xor", True)

    def __invert__(self):
        from . import bitwise_ops, logic_ops
        if self._dtype.kind in "iu":
            return bitwise_ops.invert(self)
        if self._dtype == np.bool_:
            return logic_ops.logical_not(self)
        return logic_ops.logical_not(self.astype(np.int32))

    def __lshift__(self, o):
        from . import bitwise_ops
        return bitwise_ops.left_shift(self, o)

    def __rlshift__(self, o):
        from . import bitwise_ops
        return bitwise_ops.left_shift(o, self)

    def __rshift__(self, o):
        from . import bitwise_ops
        return bitwise_ops.right_shift(self, o)

    def __rrshift__(self, o):
        from . import bitwise_ops
        return bitwise_ops.right_shift(o, self)

    def __iand__(self, o): return self._inplace_result(self & o)
    def __ior__(self, o): return self._inplace_result(self | o)
    def __ixor__(self, o): return self._inplace_result(self ^ o)
    def __ilshift__(self, o): return self._inplace_result(self << o)
    def __irshift__(self, o): return self._inplace_result(self >> o)

    def nonzero(self):
        from . import _advindex
        return _advindex.nonzero(self)

    def take(self, indices, axis=None, out=None, mode="raise"):
        from . import indexing
        return indexing.take(self, indices, axis=axis, out=out, mode=mode)

    def put(self, ind, v, mode="raise"):
        from . import indexing
        return indexing.put(self, ind, v, mode=mode)

    def compress(self, condition, axis=None, out=None):
        from . import indexing
        return indexing.compress(condition, self, axis=axis, out=out)

    # sorting (ndarray.py:2393-2412)
    def sort(self, axis=-1):
        """Sort in place."""
        from . import sorting
        self._inplace_result(sorting.sort(self, axis=axis))

    def argsort(self, axis=-1):
        from . import sorting
        return sorting.argsort(self, axis=axis)

    def searchsorted(self, v, side="left"):
        from . import sorting
        return sorting.searchsorted(self, v, side=side)

    def __iadd__(self, o): return self._inplace(o, "add_op")
    def __isub__(self, o): return self._inplace(o, "sub_op")
    def __imul__(self, o): return self._inplace(o, "mul_op")
    def __itruediv__(self, o): return self._inplace(o, "div_op")
    def __ifloordiv__(self, o): return self._inplace(o, "floor_divide_op")
    def __imod__(self, o): return self._inplace(o, "mod_op")
    def __ipow__(self, o): return self._inplace(o, "pow_op")

    def __matmul__(self, other):
        """``a @ b`` with numpy's batched semantics above 2-D (the reference's
        operator, ndarray.py:1398-1450, raises there; BASELINE's batched
        (64,1024,1024) @ (64,1024,1024) needs it)."""
        from . import linalg_top
        return linalg_top.matmul(self, other)

    def __rmatmul__(self, other):
        from . import linalg_top
        return linalg_top.matmul(other, self)

    # ------------------------------------------------------------------ reductions
    def sum(self, axis=None, dtype=None, out=None, keepdims=False):
        from . import reductions
        return reductions.sum(self, axis=axis, dtype=dtype, out=out, keepdims=keepdims)

    def prod(self, axis=None, dtype=None, out=None, keepdims=False):
        from . import reductions
        return reductions.prod(self, axis=axis, dtype=dtype, out=out, keepdims=keepdims)

    def mean(self, axis=None, dtype=None, out=None, keepdims=False):
        from . import reductions
        return reductions.mean(self, axis=axis, dtype=dtype, out=out, keepdims=keepdims)

    def var(self, axis=None, dtype=None, out=None, ddof=0, keepdims=False):
        from . import reductions
        return reductions.var(self, axis=axis, dtype=dtype, out=out, ddof=ddof, keepdims=keepdims)

    def std(self, axis=None, dtype=None, out=None, ddof=0, keepdims=False):
        from . import reductions
        return reductions.std(self, axis=axis, dtype=dtype, out=out, ddof=ddof, keepdims=keepdims)

    def max(self, axis=None, out=None, keepdims=False):
        from . import reductions
        return reductions.max(self, axis=axis, out=out, keepdims=keepdims)

    def min(self, axis=None, out=None, keepdims=False):
        from . import reductions
        return reductions.min(self, axis=axis, out=out, keepdims=keepdims)

    def argmax(self, axis=None, out=None, keepdims=False):
        from . import reductions
        return reductions.argmax(self, axis=axis, out=out, keepdims=keepdims)

    def argmin(self, axis=None, out=None, keepdims=False):
        from . import reductions
        return reductions.argmin(self, axis=axis, out=out, keepdims=keepdims)

    def any(self, axis=None, out=None, keepdims=False):
        from . import reductions
        return reductions.any(self, axis=axis, out=out, keepdims=keepdims)

    def all(self, axis=None, out=None, keepdims=False):
        from . import reductions
        return reductions.all(self, axis=axis, out=out, keepdims=keepdims)

    def cumsum(self, axis=None, dtype=None, out=None):
        from . import reductions
        return reductions.cumsum(self, axis=axis, dtype=dtype, out=out)

    def cumprod(self, axis=None, dtype=None, out=None):
        from . import reductions
        return reductions.cumprod(self, axis=axis, dtype=dtype, out=out)

    def dot(self, other, out=None):
        from . import math_ops
        return math_ops.dot(self, other, out=out)

    def clip(self, a_min=None, a_max=None):
        r = self
        if a_min is not None:
            r = r._binary_op(a_min, "max_op")
        if a_max is not None:
            r = r._binary_op(a_max, "min_op")
        return r
