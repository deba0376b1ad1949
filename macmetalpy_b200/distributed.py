"""Block-distributed arrays over the GPUs of one box (one process per GPU).

The reference is single-device (``MetalBackend``,
``src/macmetalpy/_metal_backend.py:186-204``); this is the scale-out the
B200 build adds for arrays above a size threshold.  Rows (axis 0, or the
flat index of a 1-D array) are split into contiguous blocks, one per rank,
with the remainder spread over the first ranks.  Each rank holds its block
as an ordinary ``macmetalpy_b200.ndarray`` and runs the single-GPU kernels on
it; the exchange steps are the library's own C-ABI collectives
(``mmp_allgather`` / ``mmp_allreduce`` / ``mmp_broadcast`` over NCCL on the
library stream), and every merge runs on the device:

* elementwise / ufuncs: shard-local, no collective;
* full reductions (sum, mean, var, std, max, min, argmax, argmin, nansum,
  nanmean, nanvar, nanstd, prod): one launch (``mmp_reduce_allranks``)
  reduces the shard, stores its partial into every rank's exchange block
  over NVLink (peer memory mapped at ``init``), waits for every rank's
  partial and folds them in rank order with the reduction's own arithmetic
  (var: shifted moments moved to one shift; argmax: numpy's first
  occurrence, NaN first).  Where peers cannot be mapped, the shard's
  partial goes to device memory (``mmp_reduce_partial``), an NCCL
  all-gather collects them and ``mmp_merge_partials`` folds them.  The
  result is a 0-d device array on every rank; argmax / argmin return a
  Python int, as the reference does;
* axis-1 reductions and axis-1 scans: shard-local (rows never span ranks);
* axis-0 reductions: float64 (or int64) per-column partials ->
  ``mmp_allreduce`` (SUM) -> cast on the device;
* 1-D cumsum: shard partial -> all-gather -> the merge of the lower ranks'
  partials is the carry (on the device) -> one local scan with that carry;
* matmul: A row-sharded, B broadcast in place from rank 0, C row-sharded.

No step reads a partial back to the host; kernels and collectives share one
stream, so nothing synchronises between them.  The only control-plane step is
the hand-over of the communicator id at ``init`` (``_rendezvous``).
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

__all__ = ["init", "finalize", "row_partition", "DistArray", "world", "rank", "barrier", "max_over_ranks",
           "synchronize"]

PARTIAL_BYTES = 48  # sizeof(mmp_partial)
ID_BYTES = 256  # MMP_COMM_ID_BYTES
_state = {"init": False, "rank": 0, "world": 1, "parts": None, "timeout": 120.0}


def _cb():
    from . import _cuda_backend as cb

    return cb


def init(timeout_s: float = 120.0):
    """Bind this process's GPU (``LOCAL_RANK``) and join the communicator of
    ``WORLD_SIZE`` ranks as ``RANK`` (``MASTER_ADDR`` / ``MASTER_PORT`` carry
    the id hand-over).  A rank that does not arrive within ``timeout_s``
    ends the others' ``init`` with ``RuntimeError``."""
    from ._rendezvous import exchange_root_bytes, transport

    if _state["init"]:
        return
    # in-switch reduction (NVLS) stays off: the exchanges here are small, and
    # a rank that dies while bound to a multicast object disturbs its peers
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    r = int(os.environ.get("RANK", "0"))
    w = int(os.environ.get("WORLD_SIZE", "1"))
    how = transport()  # before NCCL is opened (see _rendezvous.transport)
    cb = _cb()
    cb.CudaBackend()  # mmp_init(LOCAL_RANK)

    def make_id():
        uid = ctypes.create_string_buffer(ID_BYTES)
        cb.check(cb.lib.mmp_comm_unique_id(uid), "mmp_comm_unique_id")
        return uid.raw

    got = exchange_root_bytes(make_id, r, w, timeout_s, nbytes=ID_BYTES, how=how)
    uid = ctypes.create_string_buffer(got, ID_BYTES)
    cb.check(cb.lib.mmp_comm_init(w, r, uid, float(timeout_s)), "mmp_comm_init")
    _state.update(init=True, rank=r, world=w, timeout=float(timeout_s), peer=False)
    _state["parts"] = cb.DeviceBuffer(PARTIAL_BYTES * (w + 1))
    # the fused reduce + exchange over peer memory, when every rank can map
    # every other rank's exchange block (collective; MMP_PEER_EXCHANGE=0
    # keeps the NCCL all-gather path)
    if os.environ.get("MMP_PEER_EXCHANGE", "1") != "0":
        rc = cb.lib.mmp_comm_peer_init()
        if rc == 0:
            _state["peer"] = True
        elif rc != -4:  # MMP_E_UNSUPPORTED: stay on the NCCL path
            cb.check(rc, "mmp_comm_peer_init")


def finalize():
    """Destroy the communicator (after the stream's work is done)."""
    if not _state["init"]:
        return
    cb = _cb()
    cb.check(cb.lib.mmp_comm_destroy(), "mmp_comm_destroy")
    _state.update(init=False, rank=0, world=1, parts=None)


def world() -> int:
    return _state["world"]


def rank() -> int:
    return _state["rank"]


def synchronize(timeout_s: float = 0.0):
    """Wait for this rank's stream; a collective that cannot finish (a lost
    rank) aborts the communicator and raises instead of hanging."""
    cb = _cb()
    if _state["init"]:
        cb.check(cb.lib.mmp_comm_synchronize(float(timeout_s)), "synchronize")
    cb.CudaBackend().synchronize()


def barrier():
    """Every rank's stream has reached this point (a one-word all-reduce)."""
    from .creation import zeros

    t = zeros((1,), dtype=np.int32)
    cb = _cb()
    cb.check(cb.lib.mmp_allreduce(ctypes.c_void_p(t._ptr), ctypes.c_void_p(t._ptr), 1, cb.dtype_code(np.int32),
                                  0), "barrier")
    synchronize()


def max_over_ranks(v: float) -> float:
    """The largest of every rank's host value (device all-reduce, MAX)."""
    from .creation import array

    t = array(np.array([v], dtype=np.float64))
    cb = _cb()
    cb.check(cb.lib.mmp_allreduce(ctypes.c_void_p(t._ptr), ctypes.c_void_p(t._ptr), 1,
                                  cb.dtype_code(np.float64), 2), "max_over_ranks")
    return float(t.get()[0])


def _shard_host(obj, dtype, threshold: int):
    """The row block of host data for ``array()`` when sharding applies (a
    multi-rank job, at least ``threshold`` elements, one dimension or more),
    else None.  Every rank must pass the same data (SPMD)."""
    if not _state["init"] or _state["world"] < 2:
        return None
    host = np.asarray(obj, dtype=dtype)
    if host.ndim == 0 or host.size < threshold:
        return None
    return DistArray.from_global(host)


def _reduce_call(a, kind, axis=None, keepdims=False, ddof=0.0, dtype=None, out=None):
    """reductions.<kind>(a, axis) for a DistArray: full reductions through the
    exchange, axis 0 of a 2-D sum through the column all-reduce, other axes
    shard-local."""
    from . import reductions

    if keepdims or dtype is not None or out is not None:
        raise NotImplementedError("distributed reductions take no keepdims, dtype or out")
    if axis is not None:
        if isinstance(axis, (tuple, list)):
            if len(axis) != 1:
                raise NotImplementedError("distributed reductions over one axis or all")
            axis = axis[0]
        ax = int(axis) % a.ndim
        if ax != 0:  # along the rows of every block
            return a.map(lambda x: reductions._reduce(x, kind, ax, ddof=ddof) if kind not in ("argmax", "argmin")
                         else reductions._arg(x, kind, ax, None, False))
        if a.ndim == 2 and kind == "sum":
            return a.sum(axis=0)
        if a.ndim != 1:
            raise NotImplementedError(f"distributed {kind} along the sharded axis of a {a.ndim}-d array")
    if kind in ("var", "std", "nanvar", "nanstd"):
        return getattr(a, kind)(ddof)
    return getattr(a, kind)()


def _scan_call(a, op, axis=None, dtype=None, out=None):
    """cumsum (op 0) / cumprod (op 1) of a DistArray."""
    from . import reductions

    if dtype is not None or out is not None:
        raise NotImplementedError("distributed scans take no dtype or out")
    if a.ndim == 2 and axis is not None and int(axis) % 2 == 1:
        return a.map(lambda x: reductions._scan(x, op, 1))
    if op == 0:
        return a.cumsum(axis)
    raise NotImplementedError("distributed cumprod: along axis 1 of a 2-D array only")


def _ufunc(op_name: str, operands):
    """An elementwise op with a DistArray among its operands: the same op on
    this rank's blocks (see DistArray._operand)."""
    from .ndarray import ndarray

    lead = next(o for o in operands if isinstance(o, DistArray))
    args = [lead._operand(o) for o in operands]
    out = ndarray._elementwise(op_name, *args)
    return DistArray(out, lead.global_shape[:1] + tuple(out.shape[1:]), lead.start, lead.stop)


def row_partition(n: int, world_size: int) -> list[tuple[int, int]]:
    """Contiguous [start, stop) blocks of n rows over world_size ranks; the
    first n % world_size ranks take one extra row."""
    base, extra = divmod(int(n), int(world_size))
    out, s = [], 0
    for r in range(world_size):
        e = s + base + (1 if r < extra else 0)
        out.append((s, e))
        s = e
    return out


def _gathered_partials(local, kind: str, index_base: int) -> int:
    """All ranks' partials of ``kind`` over ``local``, rank order, on the
    device; returns the address of the first (the array holds world())."""
    from . import reductions

    cb = _cb()
    buf = _state["parts"]
    own = buf.ptr
    src = local._ensure_contiguous() if local.size else local
    cb.check(cb.lib.mmp_reduce_partial(reductions.OPC[kind], cb.dtype_code(src.dtype),
                                       ctypes.c_void_p(src._ptr if src.size else 0), int(src.size),
                                       int(index_base), ctypes.c_void_p(own)), f"partial {kind}")
    cb.check(cb.lib.mmp_allgather(ctypes.c_void_p(own), ctypes.c_void_p(own + PARTIAL_BYTES), PARTIAL_BYTES,
                                  cb.dtype_code(np.uint8)), f"allgather {kind}")
    return own + PARTIAL_BYTES


def _merge(kind: str, dtype, parts_ptr: int, nparts: int, odt, ddof: float = 0.0):
    from . import reductions

    cb = _cb()
    res = reductions._scalar_result(np.dtype(odt))
    cb.check(cb.lib.mmp_merge_partials(reductions.OPC[kind], cb.dtype_code(dtype), ctypes.c_void_p(parts_ptr),
                                       int(nparts), cb.dtype_code(odt), ctypes.c_void_p(res._buffer.ptr),
                                       float(ddof), None), f"merge {kind}")
    return res


@dataclass
class DistArray:
    """Row-block distributed array: ``local`` is this rank's block."""

    local: object
    global_shape: tuple
    start: int
    stop: int

    @property
    def dtype(self):
        return self.local.dtype

    @property
    def shape(self):
        return self.global_shape

    @classmethod
    def from_global(cls, host: np.ndarray, dtype=None) -> "DistArray":
        """Each rank uploads its own row block of a host array every rank
        can produce (e.g. from the same seed)."""
        from ._dtypes import resolve_dtype
        from .ndarray import ndarray

        host = np.asarray(host, dtype=dtype)
        s, e = row_partition(host.shape[0], world())[rank()]
        block = np.ascontiguousarray(host[s:e])
        return cls(ndarray._from_numpy(block, resolve_dtype(block.dtype)), tuple(host.shape), s, e)

    @classmethod
    def from_local(cls, local, global_rows: int) -> "DistArray":
        s, e = row_partition(global_rows, world())[rank()]
        if local.shape[0] != e - s:
            raise ValueError("local block does not match the row partition")
        return cls(local, (global_rows,) + tuple(local.shape[1:]), s, e)

    def gather(self) -> np.ndarray:
        """The whole array on the host of every rank (device all-gather of
        the padded blocks, then one read-back)."""
        from .creation import empty, zeros

        cb = _cb()
        parts = row_partition(self.global_shape[0], world())
        maxrows = max(e - s for s, e in parts)
        inner = tuple(self.global_shape[1:])
        dt = np.dtype(self.dtype)
        pad = zeros((maxrows,) + inner, dtype=dt)
        if self.local.size:
            pad[: self.stop - self.start] = self.local
        nbytes = pad.size * dt.itemsize
        allb = empty((world() * maxrows,) + inner, dtype=dt)
        cb.check(cb.lib.mmp_allgather(ctypes.c_void_p(pad._ptr), ctypes.c_void_p(allb._ptr), nbytes,
                                      cb.dtype_code(np.uint8)), "gather")
        host = allb.get().reshape((world(), maxrows) + inner)
        return np.concatenate([host[r, : e - s] for r, (s, e) in enumerate(parts)], axis=0)

    @property
    def ndim(self):
        return len(self.global_shape)

    @property
    def size(self):
        return int(np.prod(self.global_shape))

    def get(self) -> np.ndarray:
        """The whole array on the host (``gather``), as ``ndarray.get``."""
        return self.gather()

    # -- elementwise (shard-local)
    def _operand(self, o):
        """o as an operand of this rank's block: a DistArray of the same
        partition gives its block; an array spanning the global rows gives
        this rank's rows; scalars and arrays that broadcast along the rows
        pass unchanged."""
        if isinstance(o, DistArray):
            if o.global_shape[0] != self.global_shape[0] or (o.start, o.stop) != (self.start, self.stop):
                raise ValueError("distributed operands must share one row partition")
            return o.local
        shp = getattr(o, "shape", None)
        if shp is not None and len(shp) == len(self.global_shape) and shp[0] == self.global_shape[0] \
                and self.global_shape[0] > 1:
            return o[self.start:self.stop]
        return o

    def map(self, fn, *others) -> "DistArray":
        args = [self._operand(o) for o in others]
        out = fn(self.local, *args)
        return DistArray(out, self.global_shape[:1] + tuple(out.shape[1:]), self.start, self.stop)

    def __add__(self, o): return self.map(lambda a, b: a + b, o)
    def __radd__(self, o): return self.map(lambda a, b: b + a, o)
    def __sub__(self, o): return self.map(lambda a, b: a - b, o)
    def __rsub__(self, o): return self.map(lambda a, b: b - a, o)
    def __mul__(self, o): return self.map(lambda a, b: a * b, o)
    def __rmul__(self, o): return self.map(lambda a, b: b * a, o)
    def __truediv__(self, o): return self.map(lambda a, b: a / b, o)
    def __rtruediv__(self, o): return self.map(lambda a, b: b / a, o)
    def __floordiv__(self, o): return self.map(lambda a, b: a // b, o)
    def __mod__(self, o): return self.map(lambda a, b: a % b, o)
    def __pow__(self, o): return self.map(lambda a, b: a ** b, o)
    def __neg__(self): return self.map(lambda a: -a)
    def __abs__(self): return self.map(lambda a: abs(a))
    def __lt__(self, o): return self.map(lambda a, b: a < b, o)
    def __le__(self, o): return self.map(lambda a, b: a <= b, o)
    def __gt__(self, o): return self.map(lambda a, b: a > b, o)
    def __ge__(self, o): return self.map(lambda a, b: a >= b, o)
    def __matmul__(self, o): return self.matmul(o)
    def astype(self, dtype): return self.map(lambda a: a.astype(dtype))

    # -- full reductions: device partial -> all-gather -> device merge
    def _flat_base(self) -> int:
        rows = max(self.stop - self.start, 1)
        return self.start * (int(self.local.size) // rows) if self.local.size else 0

    def _full(self, kind: str, ddof: float = 0.0):
        from . import reductions

        k = kind
        if self.dtype.kind != "f" and kind.startswith("nan"):
            k = kind[3:]  # no NaN in integer arrays (nan_ops.py:132-134)
        if self.local.size == 0 and world() == 1 and k in reductions._NO_IDENTITY:
            raise ValueError(f"zero-size array to reduction operation {reductions._NO_IDENTITY[k]} "
                             "which has no identity")
        odt = reductions.out_dtype(k, self.dtype)
        if _state.get("peer"):
            # one launch: this shard's reduction, the partials stored into
            # every rank's exchange block over NVLink, the merge
            cb = _cb()
            src = self.local._ensure_contiguous() if self.local.size else self.local
            res = reductions._scalar_result(np.dtype(odt))
            cb.check(cb.lib.mmp_reduce_allranks(reductions.OPC[k], cb.dtype_code(src.dtype),
                                                ctypes.c_void_p(src._ptr if src.size else 0), int(src.size),
                                                int(self._flat_base()), cb.dtype_code(odt),
                                                ctypes.c_void_p(res._buffer.ptr), float(ddof)), f"{kind}")
            return res
        parts = _gathered_partials(self.local, k, self._flat_base())
        return _merge(k, self.dtype, parts, world(), odt, ddof)

    def sum(self, axis=None):
        from . import reductions

        if axis in (1, -1) and len(self.global_shape) == 2:
            return DistArray(reductions.sum(self.local, axis=1), self.global_shape[:1], self.start, self.stop)
        if axis == 0 and len(self.global_shape) == 2:
            cb = _cb()
            wide = np.float64 if self.dtype.kind == "f" else (np.uint64 if self.dtype.kind == "u" else np.int64)
            odt = reductions.out_dtype("sum", self.dtype)
            if self.local.size:
                # the column kernel accumulates wide already: ask for its
                # accumulator as the output (no cast pass over the block)
                from .ndarray import ndarray
                src = self.local._ensure_contiguous()
                rows, cols = src.shape
                loc = ndarray._empty((cols,), wide)
                cb.check(cb.lib.mmp_reduce_axis(reductions.OPC["sum"], cb.dtype_code(src.dtype),
                                                ctypes.c_void_p(src._ptr), 1, rows, cols, cb.dtype_code(wide),
                                                ctypes.c_void_p(loc._ptr), 0.0), "sum axis 0")
            else:
                loc = reductions.sum(self.local, axis=0).astype(wide)
            if _state.get("peer"):
                # one launch: the column partials cross NVLink into every
                # rank, summed in rank order straight into the result dtype
                from .ndarray import ndarray
                res = ndarray._empty(loc.shape, odt)
                rc = cb.lib.mmp_allreduce_sum_peer(ctypes.c_void_p(loc._ptr), ctypes.c_void_p(res._ptr),
                                                   int(loc.size), cb.dtype_code(wide), cb.dtype_code(odt))
                if rc == 0:
                    return res
                if rc != -4:  # MMP_E_UNSUPPORTED (too many columns): the same on every rank
                    cb.check(rc, "allreduce axis 0")
            cb.check(cb.lib.mmp_allreduce(ctypes.c_void_p(loc._ptr), ctypes.c_void_p(loc._ptr), int(loc.size),
                                          cb.dtype_code(wide), 0), "allreduce axis 0")
            return loc.astype(odt)
        return self._full("sum")

    def mean(self):
        return self._full("mean")

    def prod(self):
        return self._full("prod")

    def nansum(self):
        return self._full("nansum")

    def nanmean(self):
        return self._full("nanmean")

    def var(self, ddof=0):
        return self._full("var", ddof)

    def std(self, ddof=0):
        return self._full("std", ddof)

    def nanvar(self, ddof=0):
        return self._full("nanvar", ddof)

    def nanstd(self, ddof=0):
        return self._full("nanstd", ddof)

    def max(self):
        return self._full("max")

    def min(self):
        return self._full("min")

    def nanmax(self):
        return self._full("nanmax")

    def nanmin(self):
        return self._full("nanmin")

    def argmax(self) -> int:
        return int(self._full("argmax").get())

    def argmin(self) -> int:
        return int(self._full("argmin").get())

    # -- scans
    def cumsum(self, axis=None) -> "DistArray":
        from . import reductions
        from .ndarray import ndarray

        if axis in (1, -1) and len(self.global_shape) == 2:
            return DistArray(reductions.cumsum(self.local, axis=1), self.global_shape, self.start, self.stop)
        if axis in (0, -2) and len(self.global_shape) == 2:
            return self._cumsum_rows()
        if len(self.global_shape) != 1 and axis is not None:
            raise NotImplementedError("distributed cumsum: 1-D, axis 0 or 1 of 2-D, or axis=None")
        local = self.local.reshape(-1) if len(self.global_shape) != 1 else self.local
        if _state.get("peer"):
            # one collective call: the lower ranks' totals cross NVLink as peer
            # stores between the scan's own launches
            local = local._ensure_contiguous()
            odt = reductions.scan_out_dtype(self.dtype)
            res = ndarray._empty(local.shape, odt)
            cb = _cb()
            cb.check(cb.lib.mmp_scan_allranks(0, cb.dtype_code(self.dtype), ctypes.c_void_p(local._ptr),
                                              cb.dtype_code(odt), ctypes.c_void_p(res._ptr), int(local.size)),
                     "distributed cumsum")
        else:
            kind = self.dtype.kind
            carry_dt = np.float64 if kind == "f" else (np.uint64 if kind == "u" else np.int64)
            parts = _gathered_partials(local, "sum", 0)
            carry = _merge("sum", self.dtype, parts, rank(), carry_dt)  # lower ranks' total
            if local.size:
                res = reductions._scan(local, 0, None, carry_ptr=carry._buffer.ptr)
            else:
                res = ndarray._empty((0,), reductions.scan_out_dtype(self.dtype))
        if len(self.global_shape) != 1:  # axis=None of an N-d array: flat result
            n = int(np.prod(self.global_shape))
            return DistArray(res, (n,), self._flat_base(), self._flat_base() + int(local.size))
        return DistArray(res, self.global_shape, self.start, self.stop)

    def _cumsum_rows(self) -> "DistArray":
        """cumsum along axis 0 of a row-sharded 2-D array: every rank's column
        totals (the column kernel's accumulator, float64 / int64 / uint64)
        are all-gathered on the device, the rows of the ranks below this one
        summed into the column carry, and the carry added to the local
        column scan in one fused pass (float: in float64, rounded once to
        the result dtype; integers exact)."""
        from . import reductions
        from .creation import zeros
        from .ndarray import ndarray

        cb = _cb()
        kind = self.dtype.kind
        wide = np.dtype(np.float64 if kind == "f" else (np.uint64 if kind == "u" else np.int64))
        odt = reductions.scan_out_dtype(self.dtype)
        cols = int(self.global_shape[1])
        src = self.local._ensure_contiguous()
        if src.size:
            tot = ndarray._empty((cols,), wide)
            cb.check(cb.lib.mmp_reduce_axis(reductions.OPC["sum"], cb.dtype_code(src.dtype), ctypes.c_void_p(src._ptr),
                                            1, int(src.shape[0]), cols, cb.dtype_code(wide),
                                            ctypes.c_void_p(tot._ptr), 0.0), "column totals")
        else:
            tot = zeros((cols,), dtype=wide)
        allt = ndarray._empty((world() * cols,), wide)
        cb.check(cb.lib.mmp_allgather(ctypes.c_void_p(tot._ptr), ctypes.c_void_p(allt._ptr), cols,
                                      cb.dtype_code(wide)), "column totals all-gather")
        r = rank()
        if not src.size:
            res = ndarray._empty(src.shape, odt)
        elif r == 0:
            res = reductions.cumsum(src, axis=0)
        else:
            carry = reductions.sum(allt.reshape(world(), cols)[:r], axis=0)
            res = (reductions.cumsum(src, axis=0).astype(wide) + carry).astype(odt)
            res._materialize_if_lazy()
        return DistArray(res, self.global_shape, self.start, self.stop)

    # -- matmul: A row-sharded, B broadcast from rank 0
    def matmul(self, b) -> "DistArray":
        """C = A @ B with A row-sharded and B replicated: every rank passes a
        device array of B's shape and dtype; rank 0's contents are broadcast
        in place into the others' arrays (``mmp_broadcast`` on the library
        stream, so the local GEMM is ordered after it), then each rank
        multiplies its rows."""
        from . import linalg_top

        b = b._ensure_contiguous()
        if world() > 1:
            cb = _cb()
            cb.check(cb.lib.mmp_broadcast(ctypes.c_void_p(b._ptr), ctypes.c_void_p(b._ptr),
                                          int(b.size) * np.dtype(b.dtype).itemsize, cb.dtype_code(np.uint8), 0),
                     "broadcast B")
        c = linalg_top.matmul(self.local, b)
        return DistArray(c, (self.global_shape[0], b.shape[1]), self.start, self.stop)
