"""The device side of the block-distributed reductions on one GPU:

* ``mmp_reduce_partial`` over several slices of one array ("shards", empty
  ones included), written into one device array, then
  ``mmp_merge_partials`` -- checked against the oracle's restatement of the
  merge on the same slices, and against the single-GPU reduction of the
  whole array (bit-exact for integers and argmax/argmin, 1e-12 relative to
  the oracle merge and 1e-4 to the float64 result for floats);
* the zero-part merge (the carry of rank 0);
* a one-rank communicator through the C ABI (``distributed.init`` with
  WORLD_SIZE=1): DistArray reductions, cumsum with its device carry and
  gather, all on the library stream; with the peer exchange up,
  ``mmp_scan_allranks`` on both of its paths (a long aligned shard that
  exchanges its total from the tile aggregates, a ragged one that reduces
  first), cumprod through the C ABI and an empty shard.

Multi-rank runs are in test_gpu_distributed.py (two GPUs)."""

import ctypes

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

OPS = ["sum", "mean", "var", "std", "nansum", "nanmean", "nanvar", "nanstd", "max", "min", "argmax", "argmin"]
INT_OPS = ["sum", "mean", "var", "max", "min", "argmax", "argmin"]
BOUNDS = [0, 70001, 70001, 300000, 300017, 1000003]


def _device_merge(x, op, bounds, ddof=0.0):
    import macmetalpy_b200 as cp
    from macmetalpy_b200 import _cuda_backend as cb
    from macmetalpy_b200 import reductions as R

    X = cp.array(x)
    nparts = len(bounds) - 1
    parts = cp.zeros((nparts * 6,), dtype=np.int64)  # 48-byte mmp_partial each
    item = X.dtype.itemsize
    for j, (a, b) in enumerate(zip(bounds[:-1], bounds[1:])):
        cb.check(cb.lib.mmp_reduce_partial(R.OPC[op], cb.dtype_code(x.dtype), ctypes.c_void_p(X._ptr + a * item),
                                           b - a, a, ctypes.c_void_p(parts._ptr + 48 * j)), op)
    odt = R.out_dtype(op, x.dtype)
    out = cp.zeros((1,), dtype=odt)
    cb.check(cb.lib.mmp_merge_partials(R.OPC[op], cb.dtype_code(x.dtype), ctypes.c_void_p(parts._ptr), nparts,
                                       cb.dtype_code(odt), ctypes.c_void_p(out._ptr), ddof, None), op)
    return out.get()[0], X


@pytest.mark.parametrize("op", OPS)
def test_merge_float32(op):
    import macmetalpy_b200 as cp

    rng = np.random.default_rng(11)
    x = (rng.standard_normal(BOUNDS[-1]) * 5 + 300).astype(np.float32)
    if op.startswith("nan"):
        x[rng.choice(x.size, 5000, replace=False)] = np.nan
    x[[10, 700000]] = x.max() + 1 if op == "argmax" else x[[10, 700000]]  # tie across shards
    got, X = _device_merge(x, op, BOUNDS)
    parts = [O.shard_partial(op, x[a:b], a) for a, b in zip(BOUNDS[:-1], BOUNDS[1:])]
    want = O.merge_partials(op, parts)
    if op in ("argmax", "argmin"):
        assert int(got) == want == int(getattr(np, op)(x))
        assert int(got) == int(getattr(cp, op)(X))
        return
    if op in ("max", "min"):
        assert got == want
        return
    ref = {"sum": np.sum, "mean": np.mean, "var": np.var, "std": np.std, "nansum": np.nansum,
           "nanmean": np.nanmean, "nanvar": np.nanvar, "nanstd": np.nanstd}[op](x.astype(np.float64))
    # the device's per-shard partials sum float32 vectors into float64, the
    # oracle's in float64 throughout: compare both with the float64 value
    assert abs(float(got) - ref) <= 1e-4 * abs(ref), (got, ref)
    assert abs(want - ref) <= 1e-9 * abs(ref)


@pytest.mark.parametrize("op", INT_OPS)
def test_merge_int32_exact(op):
    rng = np.random.default_rng(12)
    x = rng.integers(-100, 101, BOUNDS[-1]).astype(np.int32)
    got, _ = _device_merge(x, op, BOUNDS)
    parts = [O.shard_partial(op, x[a:b], a) for a, b in zip(BOUNDS[:-1], BOUNDS[1:])]
    want = O.merge_partials(op, parts, isfloat=False)
    if op in ("mean", "var"):
        assert abs(float(got) - want) <= 1e-12 * max(abs(want), 1.0)
    else:
        assert int(got) == int(want)


def test_merge_nan_propagation_and_first_nan():
    x = np.arange(1000, dtype=np.float32)
    x[[300, 800]] = np.nan
    got, _ = _device_merge(x, "argmax", [0, 500, 1000])
    assert int(got) == 300
    got, _ = _device_merge(x, "max", [0, 500, 1000])
    assert np.isnan(got)
    got, _ = _device_merge(x, "argmin", [0, 200, 1000])
    assert int(got) == 300


def test_zero_part_merge_is_identity():
    import macmetalpy_b200 as cp
    from macmetalpy_b200 import _cuda_backend as cb

    out = cp.full((1,), 7, dtype=np.int64)
    cb.check(cb.lib.mmp_merge_partials(0, cb.dtype_code(np.int32), None, 0, cb.dtype_code(np.int64),
                                       ctypes.c_void_p(out._ptr), 0.0, None), "merge")
    assert int(out.get()[0]) == 0


def _scan_allranks_one_rank(rng):
    import macmetalpy_b200 as cp
    from macmetalpy_b200 import _cuda_backend as cb
    from macmetalpy_b200 import distributed as D

    # long aligned shard: the aggregate-total exchange between the launches
    n = (1 << 24) + 4096
    x = (rng.standard_normal(n) + 0.25).astype(np.float32)
    got = D.DistArray.from_global(x).cumsum().gather()
    ref = O.cumsum_f64(x)
    assert np.max(np.abs(got.astype(np.float64) - ref)) <= 1e-6 * np.abs(x).astype(np.float64).sum()
    xi = rng.integers(-7, 8, n).astype(np.int32)
    np.testing.assert_array_equal(D.DistArray.from_global(xi).cumsum().gather(), np.cumsum(xi, dtype=np.int64))
    # ragged and unaligned shards: reduce + exchange, then the local scan
    for m in (1, 15, 4097, (1 << 20) + 3):
        xu = rng.integers(0, 1000, m).astype(np.uint16)
        np.testing.assert_array_equal(D.DistArray.from_global(xu).cumsum().gather(),
                                      np.cumsum(xu, dtype=np.uint64))
    # cumprod through the C ABI (no DistArray method): int64 exact
    xp = rng.choice(np.array([-1, 1, 1, 2], dtype=np.int64), 5000)
    X = cp.array(xp)
    Y = cp.empty((5000,), dtype=np.int64)
    cb.check(cb.lib.mmp_scan_allranks(1, cb.dtype_code(np.int64), ctypes.c_void_p(X._ptr),
                                      cb.dtype_code(np.int64), ctypes.c_void_p(Y._ptr), 5000), "cumprod")
    np.testing.assert_array_equal(Y.get(), np.cumprod(xp))
    # an empty shard still takes part
    cb.check(cb.lib.mmp_scan_allranks(0, cb.dtype_code(np.float32), None, cb.dtype_code(np.float32), None, 0),
             "empty")
    cb.check(cb.lib.mmp_synchronize(), "sync")


def _axis0_cases(D, rng):
    """Axis-0 sums: int32 exact (int64 result), and more columns than the
    peer exchange area holds (the NCCL all-reduce path)."""
    mi = rng.integers(-50, 51, (100, 3000)).astype(np.int32)
    got = D.DistArray.from_global(mi).sum(axis=0).get()
    assert got.dtype == np.int64
    np.testing.assert_array_equal(got, mi.sum(axis=0, dtype=np.int64))
    mw = rng.standard_normal((4, 140000)).astype(np.float32)  # 140000 * 8 B > 1 MiB
    sw = D.DistArray.from_global(mw).sum(axis=0).get()
    assert sw.dtype == np.float32
    assert np.max(np.abs(sw - mw.astype(np.float64).sum(axis=0))) <= 1e-5 * np.abs(mw).sum(axis=0).max()


def test_one_rank_communicator(monkeypatch):
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    for k, v in dict(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1",
                     MASTER_PORT=str(port)).items():
        monkeypatch.setenv(k, v)
    from macmetalpy_b200 import distributed as D

    D.init(timeout_s=60)
    try:
        rng = np.random.default_rng(3)
        x = (rng.standard_normal(333333) + 0.5).astype(np.float32)
        X = D.DistArray.from_global(x)
        x64 = x.astype(np.float64)
        assert abs(float(X.sum()) - x64.sum()) <= 1e-4 * np.abs(x64).sum()
        assert abs(float(X.var()) - x64.var()) <= 1e-4 * x64.var()
        assert X.argmax() == int(np.argmax(x))
        xi = rng.integers(-100, 101, 500001).astype(np.int32)
        XI = D.DistArray.from_global(xi)
        assert int(XI.sum()) == int(xi.sum(dtype=np.int64))
        np.testing.assert_array_equal(XI.cumsum().gather(), np.cumsum(xi, dtype=np.int64))
        if D._state.get("peer"):
            _scan_allranks_one_rank(rng)
        m = rng.standard_normal((257, 129)).astype(np.float32)
        M = D.DistArray.from_global(m)
        s0 = M.sum(axis=0).get()
        assert np.max(np.abs(s0 - m.astype(np.float64).sum(axis=0))) <= 1e-4 * np.abs(m).sum(axis=0).max()
        _axis0_cases(D, rng)
        c0 = M.cumsum(axis=0).gather()
        assert np.max(np.abs(c0 - np.cumsum(m.astype(np.float64), axis=0))) <= 1e-4 * np.abs(m).sum(axis=0).max()
        mi = rng.integers(-9, 10, (300, 7)).astype(np.int32)
        np.testing.assert_array_equal(D.DistArray.from_global(mi).cumsum(axis=0).gather(),
                                      np.cumsum(mi, axis=0, dtype=np.int64))
        D.barrier()
        assert D.max_over_ranks(2.5) == 2.5
    finally:
        D.finalize()
