"""Block-distributed arrays on 2 GPUs over the library's own collectives
(C ABI), against the oracle on the whole array: sum / mean / var / argmax /
argmin / max / nansum / nanmean (the fused reduce + peer exchange when the
ranks can map each other's memory, else device partials, all-gather and
device merge), 1-D cumsum with device carries (int32 exact, float32 within
1e-4; long aligned shards and shards on different scan paths through
mmp_scan_allranks), axis-0 sums (peer all-reduce, and the NCCL all-reduce
beyond its area), axis-1 reductions and scans
(shard-local), axis-0 scans (column totals all-gathered into a carry), matmul
with B broadcast from rank 0 (a ragged K, and a rank with no rows), and the
array API on arrays sharded by set_config(shard_threshold=...).  Needs two visible GPUs; skipped
otherwise.  Ranks are child processes with a short communicator timeout;
NVLS is off (plain NCCL rings), as this test only checks results."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import oracle as O

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


def _long_and_mixed_scans(D, rank):
    """mmp_scan_allranks with long aligned shards on both ranks (each
    exchanges its total from its tile aggregates), then with rank 0 on that
    path and rank 1 on the reduce-first path, and the other way round."""
    import ctypes

    from macmetalpy_b200 import _cuda_backend as cb
    from macmetalpy_b200.creation import array, empty

    rng = np.random.default_rng(99)
    n = 2 * ((1 << 24) + 16)
    x = (rng.standard_normal(n) + 0.25).astype(np.float32)
    got = D.DistArray.from_global(x).cumsum().gather()
    ref = O.cumsum_f64(x)
    assert np.max(np.abs(got.astype(np.float64) - ref)) <= 1e-6 * np.abs(x).astype(np.float64).sum()
    for sizes in (((1 << 24) + 16, 1001), (1001, (1 << 24) + 16)):
        xs = [rng.integers(-9, 10, s).astype(np.int32) for s in sizes]
        X = array(xs[rank])
        Y = empty((sizes[rank],), dtype=np.int64)
        cb.check(cb.lib.mmp_scan_allranks(0, cb.dtype_code(np.int32), ctypes.c_void_p(X._ptr),
                                          cb.dtype_code(np.int64), ctypes.c_void_p(Y._ptr), sizes[rank]), "scan")
        want = np.cumsum(np.concatenate(xs), dtype=np.int64)
        lo = sum(sizes[:rank])
        np.testing.assert_array_equal(Y.get(), want[lo:lo + sizes[rank]])


def _threshold_sharding(D, rank):
    """set_config(shard_threshold=n): host data of at least n elements is
    uploaded as this rank's row block, and the array API works on it --
    the C1 expression, full and per-axis reductions, argmax, cumsum and
    matmul -- against numpy on the whole array; smaller arrays stay whole."""
    import macmetalpy_b200 as cp

    rng = np.random.default_rng(31)
    cp.set_config(shard_threshold=100_000)
    try:
        xs = rng.standard_normal(300_001).astype(np.float32)
        XS = cp.array(xs)
        assert isinstance(XS, D.DistArray) and XS.shape == xs.shape
        assert isinstance(cp.array(xs[:1000]), cp.ndarray)
        y = cp.sqrt(cp.abs(XS)) + cp.exp(-XS ** 2)
        assert isinstance(y, D.DistArray)
        x64 = xs.astype(np.float64)
        yref = np.sqrt(np.abs(x64)) + np.exp(-x64 ** 2)
        assert np.max(np.abs(y.get() - yref) / yref) <= 5e-7
        assert abs(float(cp.sum(y)) - yref.sum()) <= 1e-5 * yref.sum()
        assert abs(float(cp.var(XS)) - x64.var()) <= 1e-4 * x64.var()
        assert cp.argmax(XS) == int(np.argmax(xs))
        c = cp.cumsum(XS).get()
        assert np.max(np.abs(c - np.cumsum(x64))) <= 1e-6 * np.abs(x64).sum()
        m = rng.standard_normal((1000, 300)).astype(np.float32)
        M = cp.array(m)
        assert isinstance(M, D.DistArray)
        assert np.max(np.abs(cp.sum(M, axis=0).get() - m.astype(np.float64).sum(axis=0))) <= 1e-4
        assert np.max(np.abs(cp.mean(M, axis=1).get() - m.astype(np.float64).mean(axis=1))) <= 1e-5
        b = (rng.standard_normal((300, 40)) / 20).astype(np.float32)
        P = (M @ cp.array(b)).get()
        r = m.astype(np.float64) @ b.astype(np.float64)
        assert np.linalg.norm(P - r) / np.linalg.norm(r) <= 1e-5
    finally:
        cp.set_config(shard_threshold=0)


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        from macmetalpy_b200 import distributed as D
        from macmetalpy_b200.creation import array, zeros

        D.init(timeout_s=60)
        rng = np.random.default_rng(7)
        x = rng.standard_normal(1_000_003).astype(np.float32) + 0.25
        X = D.DistArray.from_global(x)
        x64 = x.astype(np.float64)
        assert abs(float(X.sum()) - x64.sum()) <= 1e-4 * np.abs(x64).sum()
        assert abs(float(X.mean()) - x64.mean()) <= 1e-4 * abs(x64.mean())
        assert abs(float(X.var()) - x64.var()) <= 1e-4 * x64.var()
        assert X.argmax() == O.argmax(x)
        assert X.argmin() == int(np.argmin(x))
        assert float(X.max()) == float(x.max())
        xt = x.copy()
        xt[[3, 900000]] = x.max() + 1  # a tie across the two shards
        assert D.DistArray.from_global(xt).argmax() == 3
        xn = x.copy()
        xn[rng.choice(x.size, 1000, replace=False)] = np.nan
        XN = D.DistArray.from_global(xn)
        assert abs(float(XN.nansum()) - np.nansum(xn.astype(np.float64))) <= 1e-4 * np.nansum(np.abs(xn))
        assert abs(float(XN.nanmean()) - np.nanmean(xn.astype(np.float64))) <= 1e-4 * abs(np.nanmean(xn))
        assert XN.argmax() == O.argmax(xn)
        # the other merge rules of the exchange
        assert abs(float(X.std()) - x64.std()) <= 1e-4 * x64.std()
        assert float(X.min()) == float(x.min())
        xn64 = xn.astype(np.float64)
        assert abs(float(XN.nanvar()) - np.nanvar(xn64)) <= 1e-4 * np.nanvar(xn64)
        assert abs(float(XN.nanstd()) - np.nanstd(xn64)) <= 1e-4 * np.nanstd(xn64)
        assert float(XN.nanmax()) == float(np.nanmax(xn))
        assert float(XN.nanmin()) == float(np.nanmin(xn))
        sg = rng.choice(np.array([-1, 1], np.int32), 200_001)
        assert int(D.DistArray.from_global(sg).prod()) == int(np.prod(sg.astype(np.int64)))
        xi2 = rng.integers(-1000, 1000, 300_001).astype(np.int32)
        xi2[[5, 250_000]] = 5000  # a tie across the shards
        XI2 = D.DistArray.from_global(xi2)
        assert XI2.argmax() == 5 and XI2.argmin() == int(np.argmin(xi2))
        xi = rng.integers(-100, 101, 3_000_017).astype(np.int32)
        XI = D.DistArray.from_global(xi)
        assert int(XI.sum()) == int(xi.sum(dtype=np.int64))
        np.testing.assert_array_equal(XI.cumsum().gather(), O.cumsum(xi))
        xf = rng.uniform(0, 1, 2_000_001).astype(np.float32)
        got = D.DistArray.from_global(xf).cumsum().gather()
        ref = O.cumsum_f64(xf)
        assert np.max(np.abs(got - ref) / ref) <= 1e-4
        if D._state.get("peer"):
            _long_and_mixed_scans(D, rank)
        _threshold_sharding(D, rank)
        m = rng.standard_normal((1001, 515)).astype(np.float32)
        M = D.DistArray.from_global(m)
        s1 = M.sum(axis=1).gather()
        assert np.max(np.abs(s1 - m.astype(np.float64).sum(axis=1))) <= 1e-4 * np.abs(m).sum(axis=1).max()
        s0 = M.sum(axis=0).get()
        assert np.max(np.abs(s0 - m.astype(np.float64).sum(axis=0))) <= 1e-4 * np.abs(m).sum(axis=0).max()
        from test_gpu_dist_merge import _axis0_cases
        _axis0_cases(D, np.random.default_rng(8))
        c1 = M.cumsum(axis=1).gather()
        assert np.max(np.abs(c1 - np.cumsum(m.astype(np.float64), axis=1))) <= 1e-3
        # axis 0 crosses the shard boundary: the lower ranks' column totals are the carry
        c0 = M.cumsum(axis=0).gather()
        assert c0.dtype == np.float32
        assert np.max(np.abs(c0 - np.cumsum(m.astype(np.float64), axis=0))) <= 1e-4 * np.abs(m).sum(axis=0).max()
        mi0 = rng.integers(-(1 << 31), (1 << 31) - 1, (777, 130), dtype=np.int64).astype(np.int32)
        ci0 = D.DistArray.from_global(mi0).cumsum(axis=0).gather()
        assert ci0.dtype == np.int64
        np.testing.assert_array_equal(ci0, np.cumsum(mi0, axis=0, dtype=np.int64))
        one = D.DistArray.from_global(np.ones((1, 9), np.int32)).cumsum(axis=0).gather()  # rank 1: no rows
        np.testing.assert_array_equal(one, np.ones((1, 9), np.int64))
        a = (rng.standard_normal((512, 384)) / 20).astype(np.float32)
        b = (rng.standard_normal((384, 640)) / 20).astype(np.float32)
        A = D.DistArray.from_global(a)
        Bl = array(b) if rank == 0 else zeros(b.shape, dtype=np.float32)
        C = A.matmul(Bl).gather()
        r = O.matmul_f64(a, b)
        assert np.linalg.norm(C - r) / np.linalg.norm(r) <= 1e-5
        # a longer, ragged K; then a one-row A, so rank 1 holds no rows and
        # still takes part in the broadcast
        for (mm, kk, nn) in ((300, 4100, 260), (1, 4096, 64)):
            a2 = (rng.standard_normal((mm, kk)) / 60).astype(np.float32)
            b2 = (rng.standard_normal((kk, nn)) / 60).astype(np.float32)
            B2 = array(b2) if rank == 0 else zeros(b2.shape, dtype=np.float32)
            C2 = D.DistArray.from_global(a2).matmul(B2).gather()
            r2 = O.matmul_f64(a2, b2)
            assert C2.shape == (mm, nn)
            assert np.linalg.norm(C2 - r2) / np.linalg.norm(r2) <= 1e-5
            np.testing.assert_array_equal(B2.get(), b2)  # the broadcast landed in place
        D.barrier()
        D.finalize()
        q.put((rank, "ok"))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_two_gpu_distributed_ops():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for r, msg in res:
        assert msg == "ok", f"rank {r}:\n{msg}"
