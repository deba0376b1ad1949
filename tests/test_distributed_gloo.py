"""Host-side logic of the block-distributed path, on CPU with world_size 2
gloo ranks: row partition, the collective helpers, and the merges of
per-shard partials (sum, var/std moments, argmax/argmin with NaN and ties,
cumsum carries) against the oracle on the whole array.  The per-shard
partials are computed here with numpy, standing in for the GPU kernels."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from macmetalpy_b200 import distributed as D


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        dist = D.init(backend="gloo", timeout_s=60)
        rng = np.random.default_rng(123)
        x = rng.standard_normal(10001) * 3 + 50
        x[4321] = np.nan if False else x[4321]
        s, e = D.row_partition(len(x), world)[rank]
        loc = x[s:e]
        # sum
        tot = D.allreduce_sum([loc.sum(), len(loc)])
        assert abs(tot[0] - x.sum()) <= 1e-9 * abs(x.sum()) and tot[1] == len(x)
        # var via shifted moments with a per-shard shift
        k = loc[0]
        parts = D.allgather_rows([len(loc), (loc - k).sum(), ((loc - k) ** 2).sum(), k])
        n, mean, m2 = D.merge_moments(parts)
        assert n == len(x)
        assert abs(mean - x.mean()) <= 1e-12 * abs(x.mean())
        assert abs(m2 / n - x.var()) <= 1e-10 * x.var()
        # argmax with a tie across the shard boundary and a NaN
        y = np.zeros(100)
        y[[10, 60, 70]] = 5.0
        ys, ye = D.row_partition(len(y), world)[rank]
        ly = y[ys:ye]
        li = int(np.argmax(ly))
        parts = D.allgather_rows([ly[li], ys + li, 1.0])
        assert D.pick_arg(parts, True) == 10
        yn = y.copy()
        yn[80] = np.nan
        yn[90] = np.nan
        lyn = yn[ys:ye]
        li = int(np.argmax(lyn))
        parts = D.allgather_rows([lyn[li], ys + li, 1.0])
        assert D.pick_arg(parts, True) == int(np.argmax(yn)) == 80
        li = int(np.argmin(ly))
        parts = D.allgather_rows([ly[li], ys + li, 1.0])
        assert D.pick_arg(parts, False) == int(np.argmin(y))
        # cumsum carry
        xi = rng.integers(-100, 101, 12345)
        cs, ce = D.row_partition(len(xi), world)[rank]
        totals = D.allgather_rows([int(xi[cs:ce].sum())], dtype=__import__("torch").int64)[:, 0]
        carry = D.exclusive_prefix([int(t) for t in totals], rank)
        local_scan = np.cumsum(xi[cs:ce]) + carry
        assert np.array_equal(local_scan, np.cumsum(xi)[cs:ce])
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as exc:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, traceback.format_exc()))


def test_row_partition():
    assert D.row_partition(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert D.row_partition(2, 4) == [(0, 1), (1, 2), (2, 2), (2, 2)]
    assert sum(e - s for s, e in D.row_partition(16384, 8)) == 16384


def test_merges_single_process():
    assert D.pick_arg([(1.0, 5, 1), (1.0, 3, 1)], True) == 3
    assert D.pick_arg([(float("nan"), 9, 1), (7.0, 1, 1)], True) == 9
    assert D.pick_arg([(0.0, 0, 0)], True) == -1
    assert D.exclusive_prefix([3, 4, 5], 2) == 7
    assert D.exclusive_prefix([2.0, 3.0], 2, prod=True) == 6.0
    x = np.arange(10.0)
    parts = [(5, (x[:5] - 0).sum(), ((x[:5]) ** 2).sum(), 0.0), (5, (x[5:] - 5).sum(), ((x[5:] - 5) ** 2).sum(), 5.0)]
    n, mean, m2 = D.merge_moments(parts)
    assert n == 10 and mean == 4.5 and abs(m2 / n - x.var()) < 1e-12


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r, msg in results:
        assert msg == "ok", f"rank {r}: {msg}"
