"""Host-side logic of the block-distributed path, on CPU with world_size-2
ranks (no GPU):

* the row partition;
* the merge rule of per-shard partials (the oracle's restatement of
  ``mmp_merge_partials``) against numpy on the whole array, with shards
  exchanged between two ``gloo`` ranks: sum, mean, var/std (shifted moments
  with a different shift per shard), nan-ops, max/min, argmax/argmin with
  ties across the shard boundary and NaNs, and the cumsum carry;
* the communicator-id hand-over (``_rendezvous``) between two processes,
  over torch's TCPStore and over a plain socket, and its timeout when rank 0
  never arrives (an error, not a hang).

The per-shard partials are computed with numpy here, standing in for the
GPU's ``mmp_reduce_partial``; the GPU tests check the device merge against
the same oracle."""

import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from macmetalpy_b200 import _rendezvous as RV
from macmetalpy_b200 import distributed as D
from oracle import oracle as O

OPS = ["sum", "mean", "var", "std", "nansum", "nanmean", "nanvar", "nanstd", "max", "min", "argmax", "argmin"]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _whole(op, x):
    x64 = x.astype(np.float64)
    return {"sum": lambda: x64.sum() if x.dtype.kind == "f" else int(x.astype(np.int64).sum()),
            "mean": lambda: x64.mean(), "var": lambda: x64.var(), "std": lambda: x64.std(),
            "nansum": lambda: np.nansum(x64), "nanmean": lambda: np.nanmean(x64),
            "nanvar": lambda: np.nanvar(x64), "nanstd": lambda: np.nanstd(x64),
            "max": lambda: x.max(), "min": lambda: x.min(),
            "argmax": lambda: int(np.argmax(x)), "argmin": lambda: int(np.argmin(x))}[op]()


def _close(got, ref, op):
    if op in ("argmax", "argmin"):
        return got == ref
    if np.isnan(ref):
        return np.isnan(got)
    return abs(got - ref) <= 1e-12 * max(abs(ref), 1.0)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
        rng = np.random.default_rng(123)
        x = (rng.standard_normal(10001) * 3 + 50).astype(np.float32)
        cases = {"plain": x}
        xn = x.copy()
        xn[[4321, 9000]] = np.nan
        cases["nan"] = xn
        tie = np.zeros(100, dtype=np.float32)
        tie[[10, 60, 70]] = 5.0
        cases["tie"] = tie
        xi = rng.integers(-100, 101, 12345).astype(np.int32)
        for name, arr in list(cases.items()) + [("int", xi)]:
            s, e = D.row_partition(len(arr), world)[rank]
            ops = OPS if arr.dtype.kind == "f" else ["sum", "mean", "var", "max", "min", "argmax", "argmin"]
            for op in ops:
                mine = O.shard_partial(op, arr[s:e], s)
                parts = [None] * world
                dist.all_gather_object(parts, mine)
                got = O.merge_partials(op, parts, isfloat=arr.dtype.kind == "f")
                ref = _whole(op, arr)
                assert _close(got, ref, op), (name, op, got, ref)
        # cumsum carry: the merge of the lower ranks' partials
        s, e = D.row_partition(len(xi), world)[rank]
        mine = O.shard_partial("sum", xi[s:e])
        parts = [None] * world
        dist.all_gather_object(parts, mine)
        carry = O.merge_partials("sum", parts[:rank], isfloat=False)
        assert np.array_equal(np.cumsum(xi[s:e], dtype=np.int64) + carry, np.cumsum(xi, dtype=np.int64)[s:e])
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, traceback.format_exc()))


def test_row_partition():
    assert D.row_partition(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert D.row_partition(2, 4) == [(0, 1), (1, 2), (2, 2), (2, 2)]
    assert sum(e - s for s, e in D.row_partition(16384, 8)) == 16384


@pytest.mark.parametrize("op", OPS)
def test_merge_rule_single_process(op):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(5000) * 7 + 1e3).astype(np.float32)
    x[[17, 4000]] = np.nan if op.startswith("nan") or op.startswith("arg") else x[[17, 4000]]
    bounds = [0, 1234, 1234, 1234, 3000, 5000]  # empty shards included
    parts = [O.shard_partial(op, x[a:b], a) for a, b in zip(bounds[:-1], bounds[1:])]
    assert _close(O.merge_partials(op, parts), _whole(op, x), op)


def test_merge_identities():
    assert O.merge_partials("sum", [], isfloat=False) == 0
    assert O.merge_partials("argmax", [O.shard_partial("argmax", np.zeros(0, np.float32))]) == -1
    nan_first = [O.shard_partial("argmax", np.array([1.0, np.nan], np.float32), 0),
                 O.shard_partial("argmax", np.array([np.nan, 9.0], np.float32), 2)]
    assert O.merge_partials("argmax", nan_first) == 1


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in results:
        assert msg == "ok", f"rank {r}: {msg}"


def _rdzv_worker(rank, world, port, transport, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), MMP_RDZV=transport)
    try:
        payload = bytes(range(128)) if rank == 0 else b"\0" * 128
        got = RV.exchange_root_bytes(payload, rank, world, timeout_s=60)
        q.put((rank, "ok" if got == bytes(range(128)) else "wrong bytes"))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("transport", ["store", "socket"])
def test_rendezvous_two_ranks(transport):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rdzv_worker, args=(r, 3, port, transport, q)) for r in range(3)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=30)
    for r, msg in results:
        assert msg == "ok", f"rank {r}: {msg}"


def test_rendezvous_times_out_without_rank0(monkeypatch):
    monkeypatch.setenv("MASTER_ADDR", "127.0.0.1")
    monkeypatch.setenv("MASTER_PORT", str(_free_port()))
    monkeypatch.setenv("MMP_RDZV", "socket")
    t0 = time.monotonic()
    with pytest.raises(TimeoutError):
        RV.exchange_root_bytes(b"\0" * 128, 1, 2, timeout_s=1.0)
    assert time.monotonic() - t0 < 10
