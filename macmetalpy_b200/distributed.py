"""Block-distributed arrays over the GPUs of one box (one process per GPU).

The reference is single-device; this is the scale-out the B200 build adds
for arrays above a size threshold.  Rows (axis 0, or the flat index of a
1-D array) are split into contiguous blocks, one per rank, with the
remainder spread over the first ranks.  Each rank holds its block as an
ordinary ``macmetalpy_b200.ndarray`` and runs the single-GPU kernels on it;
only the exchange steps use collectives (``torch.distributed`` over NCCL /
NVLink, one communicator per process group):

* elementwise / ufuncs: shard-local, no collective;
* sum / mean / nansum / nanmean: each shard's exact partial (float64 sum or
  int64 sum, and the count) -> ``all_reduce`` (SUM);
* var / std: each shard's (count, S1, S2, shift) -> ``all_gather`` -> Chan's
  pairwise merge in rank order (deterministic);
* argmax / argmin: each shard's (value, global index) -> ``all_gather`` ->
  the first extreme wins, NaN first (numpy's rule);
* max / min: ``all_gather`` of the shard extremes (NaN propagates);
* axis-1 reductions and axis-1 cumsum: shard-local (rows never span ranks);
* axis-0 reductions: float64 per-column partials -> ``all_reduce`` (SUM);
* 1-D cumsum: shard totals -> ``all_gather`` -> exclusive prefix of the
  lower ranks -> one local scan with that carry (one read, one write);
* matmul: A row-sharded, B broadcast from rank 0 (``broadcast``), C
  row-sharded.

The library and torch share one current stream, so kernels and NCCL
collectives are ordered on the device without host synchronisation.  The
merge helpers (``merge_moments``, ``pick_arg``, ``exclusive_prefix``,
``row_partition``) are pure functions, tested on CPU with ``gloo`` ranks.
"""

from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass

import numpy as np

__all__ = [
    "init", "row_partition", "DistArray", "merge_moments", "pick_arg", "exclusive_prefix", "world", "rank",
]

_state = {"init": False, "dist": None, "device": "cpu"}


def init(backend: str | None = None, timeout_s: float = 120.0):
    """Join (or create) the default process group and bind this process's
    GPU.  Uses the RANK / WORLD_SIZE / LOCAL_RANK / MASTER_* environment."""
    import datetime

    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = {}
        if backend == "nccl":
            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    _state["dist"] = dist
    _state["init"] = True
    _state["device"] = "cuda" if dist.get_backend() == "nccl" else "cpu"
    if _state["device"] == "cuda":
        from . import _cuda_backend as cb

        cb.CudaBackend()
        cur = torch.cuda.current_stream()
        if cur.cuda_stream == 0:
            # torch is on the legacy default stream: make the library's own
            # (non-blocking) stream torch's current stream instead
            h = ctypes.c_void_p()
            cb.check(cb.lib.mmp_get_stream(ctypes.byref(h)), "get stream")
            torch.cuda.set_stream(torch.cuda.ExternalStream(h.value, device=torch.cuda.current_device()))
        else:
            cb.check(cb.lib.mmp_set_stream(ctypes.c_void_p(cur.cuda_stream)), "set stream")
    return dist


def world() -> int:
    d = _state["dist"]
    return d.get_world_size() if d is not None and d.is_initialized() else 1


def rank() -> int:
    d = _state["dist"]
    return d.get_rank() if d is not None and d.is_initialized() else 0


# ---------------------------------------------------------------------------
# pure helpers (no GPU)
# ---------------------------------------------------------------------------


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


def merge_moments(parts) -> tuple[float, float, float]:
    """Merge per-shard (count, S1, S2, shift) with S1 = sum(x - shift) and
    S2 = sum((x - shift)^2) into (count, mean, M2) by Chan et al.'s pairwise
    update, in rank order."""
    n_tot, mean_tot, m2_tot = 0.0, 0.0, 0.0
    for cnt, s1, s2, k in parts:
        cnt = float(cnt)
        if cnt == 0:
            continue
        mean = k + s1 / cnt
        m2 = max(s2 - s1 * s1 / cnt, 0.0)
        if n_tot == 0:
            n_tot, mean_tot, m2_tot = cnt, mean, m2
            continue
        delta = mean - mean_tot
        n_new = n_tot + cnt
        mean_tot = mean_tot + delta * cnt / n_new
        m2_tot = m2_tot + m2 + delta * delta * n_tot * cnt / n_new
        n_tot = n_new
    return n_tot, mean_tot, m2_tot


def pick_arg(parts, maximum: bool = True) -> int:
    """Global argmax/argmin from per-shard (value, global_index, present):
    the larger (smaller) value wins, NaN beats every number, ties keep the
    lower index (numpy's first occurrence)."""
    best = None
    for v, i, present in parts:
        if not present:
            continue
        v = float(v)
        i = int(i)
        if best is None:
            best = (v, i)
            continue
        bv, bi = best
        vn, bn = math.isnan(v), math.isnan(bv)
        if vn or bn:
            if vn and bn:
                take = i < bi
            else:
                take = vn
        elif v != bv:
            take = (v > bv) if maximum else (v < bv)
        else:
            take = i < bi
        if take:
            best = (v, i)
    return -1 if best is None else best[1]


def exclusive_prefix(totals, r: int, prod: bool = False):
    """Combination of the totals of ranks 0..r-1 (the carry of rank r)."""
    acc = 1 if prod else 0
    for t in totals[:r]:
        acc = acc * t if prod else acc + t
    return acc


# ---------------------------------------------------------------------------
# collectives on small host vectors
# ---------------------------------------------------------------------------


def _t(x, dtype):
    import torch

    return torch.as_tensor(np.asarray(x), dtype=dtype, device=_state["device"])


def allgather_rows(vec, dtype=None) -> np.ndarray:
    """(world, len(vec)) array of every rank's ``vec``."""
    import torch

    dist = _state["dist"]
    dt = dtype or torch.float64
    t = _t(vec, dt).reshape(-1)
    out = [torch.empty_like(t) for _ in range(world())]
    dist.all_gather(out, t)
    return np.stack([o.cpu().numpy() for o in out])


def allreduce_sum(vec, dtype=None) -> np.ndarray:
    import torch

    dist = _state["dist"]
    t = _t(vec, dtype or torch.float64).reshape(-1)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.cpu().numpy()


# ---------------------------------------------------------------------------
# distributed array
# ---------------------------------------------------------------------------


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
        from .creation import array

        host = np.asarray(host)
        s, e = row_partition(host.shape[0], world())[rank()]
        return cls(array(host[s:e], dtype=dtype), tuple(host.shape), s, e)

    @classmethod
    def from_local(cls, local, global_rows: int) -> "DistArray":
        s, e = row_partition(global_rows, world())[rank()]
        if local.shape[0] != e - s:
            raise ValueError("local block does not match the row partition")
        return cls(local, (global_rows,) + tuple(local.shape[1:]), s, e)

    def gather(self) -> np.ndarray:
        """The whole array on the host (every rank)."""
        parts = row_partition(self.global_shape[0], world())
        maxrows = max(e - s for s, e in parts)
        loc = self.local.get()
        pad = np.zeros((maxrows,) + loc.shape[1:], dtype=loc.dtype)
        pad[: loc.shape[0]] = loc
        rows = allgather_rows(pad.reshape(-1).view(np.uint8), dtype=_uint8())
        out = []
        for (s, e), r in zip(parts, rows):
            out.append(r.view(loc.dtype).reshape((maxrows,) + loc.shape[1:])[: e - s])
        return np.concatenate(out, axis=0)

    # -- elementwise (shard-local)
    def map(self, fn, *others) -> "DistArray":
        args = [o.local if isinstance(o, DistArray) else o for o in others]
        return DistArray(fn(self.local, *args), self.global_shape, self.start, self.stop)

    def __add__(self, o): return self.map(lambda a, b: a + b, o)
    def __sub__(self, o): return self.map(lambda a, b: a - b, o)
    def __mul__(self, o): return self.map(lambda a, b: a * b, o)
    def __truediv__(self, o): return self.map(lambda a, b: a / b, o)
    def __floordiv__(self, o): return self.map(lambda a, b: a // b, o)
    def __mod__(self, o): return self.map(lambda a, b: a % b, o)

    # -- reductions
    def _partial(self, kind):
        from . import reductions

        _, p = reductions._reduce(self.local, kind, None, partial=True)
        return p

    def sum(self, axis=None):
        from . import reductions

        if axis in (1, -1) and len(self.global_shape) == 2:
            return DistArray(reductions.sum(self.local, axis=1), self.global_shape[:1], self.start, self.stop)
        if axis == 0 and len(self.global_shape) == 2:
            from .creation import asarray
            loc = reductions.sum(self.local.astype(np.float64) if self.dtype.kind == "f" else self.local, axis=0)
            tot = allreduce_sum(loc.get(), _torch_dt(loc.dtype))
            return asarray(tot.astype(reductions.out_dtype("sum", self.dtype)))
        p = self._partial("sum")
        if self.dtype.kind in "iub":
            return int(allreduce_sum([p.ival], _int64())[0])
        return float(allreduce_sum([p.s1])[0])

    def mean(self):
        p = self._partial("sum")
        v = allreduce_sum([p.s1 if self.dtype.kind == "f" else float(p.ival), float(p.count)])
        return v[0] / v[1]

    def nansum(self):
        p = self._partial("nansum")
        return float(allreduce_sum([p.s1])[0])

    def nanmean(self):
        p = self._partial("nanmean")
        v = allreduce_sum([p.s1, float(p.count)])
        return v[0] / v[1] if v[1] > 0 else float("nan")

    def var(self, ddof=0):
        p = self._partial("var")
        parts = allgather_rows([float(p.count), p.s1, p.s2, p.shift])
        n, _, m2 = merge_moments(parts)
        return m2 / max(n - ddof, 0) if n - ddof > 0 else float("inf") if m2 > 0 else float("nan")

    def std(self, ddof=0):
        return math.sqrt(self.var(ddof))

    def _arg(self, kind):
        n_local = int(np.prod(self.local.shape))
        if n_local:
            from . import reductions

            li = int(getattr(reductions, kind)(self.local))
            v = float(self.local.reshape(-1)[li].get())
            gi = self.start * (n_local // max(self.stop - self.start, 1)) + li
            row = [v, float(gi), 1.0]
        else:
            row = [0.0, -1.0, 0.0]
        parts = allgather_rows(row)
        return pick_arg(parts, maximum=(kind == "argmax"))

    def argmax(self):
        return self._arg("argmax")

    def argmin(self):
        return self._arg("argmin")

    def max(self):
        from . import reductions

        v = float(reductions.max(self.local).get()) if self.local.size else -math.inf
        vals = allgather_rows([v])[:, 0]
        return float(np.max(vals)) if not np.isnan(vals).any() else float("nan")

    def min(self):
        from . import reductions

        v = float(reductions.min(self.local).get()) if self.local.size else math.inf
        vals = allgather_rows([v])[:, 0]
        return float(np.min(vals)) if not np.isnan(vals).any() else float("nan")

    # -- scans
    def cumsum(self, axis=None) -> "DistArray":
        from . import _cuda_backend as cb
        from . import reductions
        from .creation import array

        if axis in (1, -1) and len(self.global_shape) == 2:
            return DistArray(reductions.cumsum(self.local, axis=1), self.global_shape, self.start, self.stop)
        if len(self.global_shape) != 1:
            raise NotImplementedError("distributed cumsum: 1-D or axis=1 of 2-D")
        isint = self.dtype.kind in "iub"
        if isint:
            tot = int(reductions.sum(self.local).get()) if self.local.size else 0
            totals = allgather_rows([tot], _int64())[:, 0]
            carry = int(exclusive_prefix([int(t) for t in totals], rank()))
            c = array(np.array([carry], dtype=np.uint64 if self.dtype.kind == "u" else np.int64))
        else:
            p = self._partial("sum") if self.local.size else None
            totals = allgather_rows([p.s1 if p else 0.0])[:, 0]
            c = array(np.array([exclusive_prefix(list(totals), rank())], dtype=np.float64))
        res = reductions._scan(self.local, 0, None, carry_ptr=c._ptr) if self.local.size else self.local
        cb.CudaBackend()
        return DistArray(res, self.global_shape, self.start, self.stop)

    # -- matmul: A row-sharded, B broadcast from rank 0
    def matmul(self, b) -> "DistArray":
        """C = A @ B with A row-sharded and B replicated: every rank passes a
        device array of B's shape and dtype; rank 0's contents are broadcast
        into the others (NCCL), then each rank multiplies its rows."""
        import torch

        from . import linalg_top

        dist = _state["dist"]
        if world() > 1:
            tb = torch.as_tensor(b, device="cuda")
            dist.broadcast(tb, src=0)
        c = linalg_top.matmul(self.local, b)
        return DistArray(c, (self.global_shape[0], b.shape[1]), self.start, self.stop)


def _torch_dt(dt):
    import torch

    return {np.dtype(np.float64): torch.float64, np.dtype(np.float32): torch.float32,
            np.dtype(np.int64): torch.int64, np.dtype(np.uint64): torch.int64}.get(np.dtype(dt), torch.float64)


def _int64():
    import torch

    return torch.int64


def _uint8():
    import torch

    return torch.uint8
