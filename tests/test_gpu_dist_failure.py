"""Failure detection of the distributed exchanges on 2 GPUs, without a GPU
fault: rank 1 stays alive (its exchange block stays mapped) but never joins
the call; rank 0's exchange -- the fused reduce + exchange, the scan's
carry exchange, the axis-0 column all-reduce -- waits for rank 1's flag,
gives up after its bounded wait (2 s of device time), sets device error 8
and returns, and rank 0's synchronize raises instead of hanging.  Both
ranks then finish normally.  Needs two visible GPUs; skipped otherwise.
NVLS is off; the exchanges use plain peer stores."""

import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, port, q, done, op):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        from macmetalpy_b200 import distributed as D

        D.init(timeout_s=60)
        if not D._state.get("peer"):
            q.put((rank, "skip: no peer exchange"))
            done.wait(60)
            D.finalize()
            return
        if op == "sum_axis0":
            X = D.DistArray.from_global(np.ones((64, 1000), dtype=np.float32))
        else:
            X = D.DistArray.from_global(np.arange(1 << 20, dtype=np.float32))
        D.barrier()
        if rank == 0:
            t0 = time.monotonic()
            r = X.sum() if op == "sum" else (X.cumsum() if op == "cumsum" else X.sum(axis=0))
            try:
                D.synchronize()
                got = "no error"
            except RuntimeError as e:
                got = str(e)
            dt = time.monotonic() - t0
            ok = "error code 8" in got and dt < 30
            q.put((rank, "ok" if ok else f"expected device error 8 within 30 s, got {got!r} after {dt:.1f} s"))
            del r
            done.set()
        else:
            done.wait(60)  # alive, its block mapped, but it never joins
            q.put((rank, "ok"))
        D.finalize()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
        done.set()


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("op", ["sum", "cumsum", "sum_axis0"])
def test_rank_that_never_joins_ends_in_an_error(op):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    port = _port()
    ps = [ctx.Process(target=_rank_main, args=(r, port, q, done, op)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for r, msg in res:
        if msg.startswith("skip"):
            pytest.skip(msg)
        assert msg == "ok", f"rank {r}:\n{msg}"
