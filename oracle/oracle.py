"""CPU oracle for the macmetalpy_b200 hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs
(``cpu_baseline`` and ``--impl reference``) may import this module, and only
as the checker / the timed CPU baseline.  The product path
(``macmetalpy_b200``) never imports it and has no CPU fallback.

It restates, with numpy, what the reference computes on its CPU path for
each op of the hot path (the reference's Metal path cannot run on Linux; its
CPU branch is plain numpy dispatch, ``ndarray.py:960-1159``).  Each function
cites the reference code it follows.  Parity is pinned: ``tests/
test_oracle_golden.py`` checks every function against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference itself.

For float reductions and scans the target tolerance is stated against a
float64-accumulated result (the ``*_f64`` helpers), because the reference's
float32 CPU results drift at the BASELINE sizes (a sequential float32
``cumsum`` of 2^30 values in U(0,1) stalls once the prefix passes 2^24).
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "resolve_dtype", "c1_expression", "add", "floor_divide", "mod", "logaddexp", "broadcast_add",
    "reduce_sum", "reduce_mean", "reduce_var", "argmax", "argmax_axis", "nansum", "nanmean",
    "cumsum", "matmul", "sum_f64", "mean_f64", "var_f64", "cumsum_f64", "matmul_f64", "ulp_error",
    "logical", "logical_not", "predicate", "isclose", "allclose", "array_equal", "count_nonzero",
    "nan_to_num", "bitwise", "invert", "op_and", "op_or", "op_xor", "op_invert", "op_shift",
    "nanprod", "nancumsum", "nancumprod", "nanvar", "nanstd", "nanargmax", "nanargmin",
    "sort", "argsort", "searchsorted",
    "getitem", "setitem", "take", "take_along_axis", "nonzero", "flatnonzero", "argwhere", "compress",
    "extract", "put", "putmask",
]


def resolve_dtype(dtype, float64_behavior: str = "cpu_fallback", default_float: str = "float32"):
    """``_dtypes.resolve_dtype`` (src/macmetalpy/_dtypes.py:77-136)."""
    if dtype is None:
        return np.dtype(default_float)
    dt = np.dtype(dtype)
    if dt == np.float64:
        return np.dtype(default_float) if float64_behavior == "downcast" else dt
    if dt == np.int8:
        return np.dtype(np.int16)
    if dt == np.uint8:
        return np.dtype(np.uint16)
    return dt


# ---------------------------------------------------------------- elementwise


def c1_expression(x):
    """``sqrt(abs(x)) + exp(-x**2)`` as the reference evaluates it op by op
    (math_ops.sqrt/exp ``math_ops.py:15-34`` -> ``_unary_op`` CPU branch
    ``ndarray.py:1161-1180``; ``x**2`` -> ``__pow__`` ``ndarray.py:1371``)."""
    x = np.asarray(x)
    return np.sqrt(np.abs(x)) + np.exp(-(x * x))


def add(a, b):
    """``ufunc_ops.add`` (ufunc_ops.py:38-45) -> numpy add."""
    return np.add(a, b)


def floor_divide(a, b):
    """``ufunc_ops.floor_divide`` (ufunc_ops.py:101-108) -> numpy floor_divide
    (floor semantics; integer division by zero gives 0)."""
    with np.errstate(all="ignore"):
        return np.floor_divide(a, b)


def mod(a, b):
    """``math_ops.mod`` / ``ndarray.__mod__`` (math_ops.py:540-548,
    ndarray.py:2525-2530): ``x1 - floor_divide(x1, x2) * x2``, each step a
    numpy op in the array dtype (not ``np.remainder``)."""
    with np.errstate(all="ignore"):
        fd = np.floor_divide(a, b)
        return a - fd * b


def logaddexp(a, b):
    """``ufunc_ops.logaddexp`` (ufunc_ops.py:238-244) -> numpy logaddexp."""
    return np.logaddexp(a, b)


def broadcast_add(a, b):
    """``_binary_op`` with ``needs_broadcast`` (ndarray.py:1062-1065): numpy
    broadcasting add."""
    return np.add(a, b)


# ---------------------------------------------------------------- reductions


def reduce_sum(a, axis=None):
    """``reductions.sum`` CPU branch (reductions.py:86-100): ``np.sum`` --
    int32 accumulates and returns int64."""
    return np.sum(a, axis=axis)


def reduce_mean(a, axis=None):
    """``reductions.mean`` CPU branch (reductions.py:128-150): ``np.mean``."""
    return np.mean(a, axis=axis)


def reduce_var(a, axis=None, ddof=0):
    """``reductions.var`` CPU branch (reductions.py:540-556): ``np.var``."""
    return np.var(a, axis=axis, ddof=ddof)


def argmax(a):
    """``reductions.argmax(axis=None)`` (reductions.py:381-418): a Python
    int, first occurrence, the first NaN wins (numpy)."""
    return int(np.argmax(a))


def argmax_axis(a, axis):
    """``reductions.argmax(axis=k)`` -> ``_reduce_axis(..., out_dtype=int32)``
    (reductions.py:410, ndarray.py:2015-2035): numpy argmax cast to int32."""
    return np.asarray(np.argmax(a, axis=axis), dtype=np.int32)


def nansum(a, axis=None):
    """``nan_ops.nansum`` (nan_ops.py:112-168) -> ``np.nansum``."""
    return np.nansum(a, axis=axis)


def nanmean(a, axis=None):
    """``nan_ops.nanmean`` (nan_ops.py:379-432) -> ``np.nanmean`` (NaN when
    a slice holds no number)."""
    with np.errstate(all="ignore"):
        import warnings

        with warnings.catch_warnings():
            warnings.simplefilter("ignore", RuntimeWarning)
            return np.nanmean(a, axis=axis)


def cumsum(a, axis=None):
    """``reductions.cumsum`` CPU branch (reductions.py:661-681):
    ``np.cumsum`` (int32 -> int64)."""
    return np.cumsum(a, axis=axis)


def matmul(a, b):
    """``linalg_top.matmul`` CPU branch (linalg_top.py:94-111): ``np.matmul``
    (float16 in, float16 out)."""
    return np.matmul(a, b)


# ---------------------------------------------------------------- float64 references


def sum_f64(a, axis=None):
    return np.sum(np.asarray(a, dtype=np.float64), axis=axis)


def mean_f64(a, axis=None):
    return np.mean(np.asarray(a, dtype=np.float64), axis=axis)


def var_f64(a, axis=None, ddof=0):
    return np.var(np.asarray(a, dtype=np.float64), axis=axis, ddof=ddof)


def cumsum_f64(a, axis=None):
    return np.cumsum(np.asarray(a, dtype=np.float64), axis=axis)


def matmul_f64(a, b):
    return np.matmul(np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64))


def ulp_error(got, ref64) -> np.ndarray:
    """|got - ref| in units of the float32 ulp at the float32-rounded
    reference (the <= 2 ulp bar for transcendentals)."""
    got = np.asarray(got, dtype=np.float32)
    ref32 = np.asarray(ref64, dtype=np.float32)
    spacing = np.spacing(np.abs(ref32)).astype(np.float64)
    spacing[spacing == 0] = np.finfo(np.float32).tiny
    err = np.abs(got.astype(np.float64) - np.asarray(ref64, dtype=np.float64)) / spacing
    both_nan = np.isnan(got) & np.isnan(ref32)
    same_inf = np.isinf(got) & np.isinf(ref32) & (np.sign(got) == np.sign(ref32))
    err[both_nan | same_inf] = 0.0
    return err


# ------------------------------------------- comparison / logic / bitwise


def logical(name, a, b):
    """``logic_ops.logical_and/or/xor`` (logic_ops.py:45-66): the CPU branch
    of ``_logical_binary`` calls ``np.logical_*`` on the operands as they are
    (logic_ops.py:32-37)."""
    return getattr(np, name)(a, b)


def logical_not(a):
    """``logic_ops.logical_not`` (logic_ops.py:53-61) -> ``np.logical_not``."""
    return np.logical_not(a)


def predicate(name, a):
    """``isnan/isinf/isfinite`` (math_ops.py:558-577) and ``signbit``
    (ufunc_ops.py:352-354): ``_unary_predicate_op``'s CPU branch
    (ndarray.py:1255-1273) calls the numpy predicate."""
    return getattr(np, name)(a)


def isclose(a, b, rtol=1e-5, atol=1e-8, equal_nan=False):
    """``math_ops.isclose`` CPU branch (math_ops.py:646-648) -> ``np.isclose``."""
    return np.isclose(a, b, rtol=rtol, atol=atol, equal_nan=equal_nan)


def allclose(a, b, rtol=1e-5, atol=1e-8, equal_nan=False):
    """``math_ops.allclose`` (math_ops.py:663-673): Python bool."""
    return bool(np.allclose(a, b, rtol=rtol, atol=atol, equal_nan=equal_nan))


def array_equal(a, b, equal_nan=False):
    """``math_ops.array_equal`` (math_ops.py:676-690): False on a shape
    mismatch, else ``np.array_equal``; Python bool."""
    a, b = np.asarray(a), np.asarray(b)
    if a.shape != b.shape:
        return False
    return bool(np.array_equal(a, b, equal_nan=equal_nan))


def count_nonzero(a, axis=None, keepdims=False):
    """``math_ops.count_nonzero`` (math_ops.py:693-705): Python int without
    an axis, else an intp array."""
    r = np.count_nonzero(a, axis=axis, keepdims=keepdims)
    if axis is None and not keepdims:
        return int(r)
    return np.asarray(r)


def nan_to_num(x, nan=0.0, posinf=None, neginf=None):
    """``math_ops.nan_to_num`` (math_ops.py:580-636): numpy's replacement,
    posinf/neginf defaulting to the dtype's finite extremes."""
    x = np.asarray(x)
    if x.dtype.kind != "f":
        return x.copy()
    fi = np.finfo(x.dtype)
    return np.nan_to_num(x, copy=True, nan=nan, posinf=fi.max if posinf is None else posinf,
                         neginf=fi.min if neginf is None else neginf)


def bitwise(name, a, b):
    """``bitwise_ops.bitwise_and/or/xor/left_shift/right_shift``
    (bitwise_ops.py:35-56, 58-95): both operands cast to int32, then the
    numpy function (CPU branch :37-45); int32 result."""
    return getattr(np, name)(np.asarray(a).astype(np.int32), np.asarray(b).astype(np.int32))


def invert(a):
    """``bitwise_ops.invert`` (bitwise_ops.py:70-82): ``~int32(a)``."""
    return np.invert(np.asarray(a).astype(np.int32))


def _bool_other(o):
    return o if isinstance(o, np.ndarray) else np.asarray(o).astype(np.bool_)


def op_and(a, b):
    """``ndarray.__and__`` (ndarray.py:1670-1674): int32 bitwise for integer
    arrays, else ``_boolean_op``'s CPU branch ``np.logical_and``
    (ndarray.py:1588-1600) with a non-array operand taken as bool."""
    a = np.asarray(a)
    return bitwise("bitwise_and", a, b) if a.dtype.kind in "iu" else np.logical_and(a, _bool_other(b))


def op_or(a, b):
    """``ndarray.__or__`` (ndarray.py:1676-1680)."""
    a = np.asarray(a)
    return bitwise("bitwise_or", a, b) if a.dtype.kind in "iu" else np.logical_or(a, _bool_other(b))


def op_xor(a, b):
    """``ndarray.__xor__`` (ndarray.py:2578-2583)."""
    a = np.asarray(a)
    return bitwise("bitwise_xor", a, b) if a.dtype.kind in "iu" else np.logical_xor(a, _bool_other(b))


def op_invert(a):
    """``ndarray.__invert__`` (ndarray.py:1682-1703): integers ->
    ``bitwise_ops.invert``; bool -> the ``bool_not_op`` kernel (logical not,
    ``_kernels.py:968-972``); other dtypes -> ``not_op`` on the int32 cast,
    read back as bool (``_kernels.py:889-894``, ``ndarray.py:1696-1703``).
    The bool and float cases have no CPU branch in the reference; this is
    what those kernels compute."""
    a = np.asarray(a)
    if a.dtype.kind in "iu":
        return invert(a)
    if a.dtype == np.bool_:
        return np.logical_not(a)
    return np.logical_not(a.astype(np.int32))


def op_shift(name, a, b):
    """``ndarray.__lshift__/__rshift__`` (ndarray.py:2549-2565) ->
    ``bitwise_ops.left_shift/right_shift``."""
    return bitwise(name, a, b)


# ------------------------------------------------- remaining NaN-aware ops


def _isfloat(a):
    return np.asarray(a).dtype.kind == "f"


def nanprod(a, axis=None):
    """``nan_ops.nanprod`` (nan_ops.py:171-214): float -> ``np.nanprod``
    (CPU branch :191-199); integers -> ``reductions.prod`` (``np.prod``)."""
    return np.nanprod(a, axis=axis) if _isfloat(a) else np.prod(a, axis=axis)


def nancumsum(a, axis=None):
    """``nan_ops.nancumsum`` (nan_ops.py:215-241): float -> ``np.nancumsum``;
    integers -> ``reductions.cumsum`` (int32 -> int64)."""
    return np.nancumsum(a, axis=axis) if _isfloat(a) else np.cumsum(a, axis=axis)


def nancumprod(a, axis=None):
    """``nan_ops.nancumprod`` (nan_ops.py:244-270)."""
    return np.nancumprod(a, axis=axis) if _isfloat(a) else np.cumprod(a, axis=axis)


def nanvar(a, axis=None, ddof=0):
    """``nan_ops.nanvar`` (nan_ops.py:484-559): float -> ``np.nanvar`` (CPU
    branch :503-509); integers -> ``reductions.var`` (``np.var``)."""
    return np.nanvar(a, axis=axis, ddof=ddof) if _isfloat(a) else np.var(a, axis=axis, ddof=ddof)


def nanstd(a, axis=None, ddof=0):
    """``nan_ops.nanstd`` (nan_ops.py:444-481): ``np.nanstd``."""
    return np.nanstd(a, axis=axis, ddof=ddof) if _isfloat(a) else np.std(a, axis=axis, ddof=ddof)


def _nanarg(fn_nan, fn_int, a, axis):
    if not _isfloat(a):
        return int(fn_int(a)) if axis is None else np.asarray(fn_int(a, axis=axis), dtype=np.int32)
    r = fn_nan(a, axis=axis)
    return int(r) if axis is None else np.asarray(r)


def nanargmax(a, axis=None):
    """``nan_ops.nanargmax`` (nan_ops.py:562-584): float -> ``np.nanargmax``
    (Python int without an axis, numpy's int64 with one; ValueError on an
    all-NaN slice); integers -> ``reductions.argmax`` (int32 with an axis)."""
    return _nanarg(np.nanargmax, np.argmax, a, axis)


def nanargmin(a, axis=None):
    """``nan_ops.nanargmin`` (nan_ops.py:587-612)."""
    return _nanarg(np.nanargmin, np.argmin, a, axis)


# ------------------------------------------------------ sort / searchsorted


def sort(a, axis=-1):
    """``sorting.sort`` CPU branch (sorting.py:22-35): ``np.sort``.  Values
    do not depend on the sort kind (NaN last)."""
    return np.sort(a, axis=axis)


def argsort(a, axis=-1):
    """``sorting.argsort`` CPU branch (sorting.py:41-54): ``np.argsort``.
    The reference passes ``kind=None`` (numpy's unstable default, ties in an
    unspecified order); this restatement uses ``kind="stable"``, which agrees
    with it wherever there are no ties and defines the tie order the device
    sort guarantees."""
    return np.argsort(a, axis=axis, kind="stable")


def searchsorted(a, v, side="left", sorter=None):
    """``sorting.searchsorted`` fallback (sorting.py:270-272):
    ``np.searchsorted`` (numpy order, NaN last; common dtype; int64)."""
    return np.searchsorted(a, v, side=side, sorter=sorter)


# ------------------------------------------------------ advanced indexing


def getitem(a, key):
    """``ndarray.__getitem__`` with an advanced key (ndarray.py:874-941): the
    CPU branch indexes the host copy with numpy."""
    return np.asarray(a)[key]


def setitem(a, key, value):
    """``ndarray.__setitem__`` advanced branch (ndarray.py:948-957):
    ``np_data[key] = value`` on a copy (returned)."""
    b = np.array(a, copy=True)
    b[key] = value
    return b


def take(a, indices, axis=None, mode="raise"):
    """``indexing.take`` (indexing.py:24-91) -> ``np.take``."""
    return np.take(a, indices, axis=axis, mode=mode)


def take_along_axis(a, indices, axis):
    """``indexing.take_along_axis`` (indexing.py:94-100)."""
    return np.take_along_axis(a, indices, axis)


def nonzero(a):
    """``indexing.nonzero`` (indexing.py:370-374) -> ``np.nonzero``."""
    return np.nonzero(a)


def flatnonzero(a):
    """``indexing.flatnonzero`` (indexing.py:377-381)."""
    return np.flatnonzero(a)


def argwhere(a):
    """``indexing.argwhere`` (indexing.py:384-391)."""
    return np.argwhere(a)


def compress(condition, a, axis=None):
    """``indexing.compress`` (indexing.py:221-231)."""
    return np.compress(condition, a, axis=axis)


def extract(condition, a):
    """``indexing.extract`` (indexing.py:242-251)."""
    return np.extract(condition, a)


def put(a, ind, v, mode="raise"):
    """``indexing.put`` (indexing.py:103-163): ``np.put`` on a copy."""
    b = np.array(a, copy=True)
    np.put(b, ind, v, mode=mode)
    return b


def putmask(a, mask, values):
    """``indexing.putmask`` (indexing.py:179-189): ``np.putmask`` on a copy."""
    b = np.array(a, copy=True)
    np.putmask(b, mask, values)
    return b


# ---------------------------------------------------------------- order statistics
def median(a, axis=None, keepdims=False):
    """``reductions.median`` (reductions.py:627-641): ``np.median`` on the
    host copy."""
    return np.median(a, axis=axis, keepdims=keepdims)


def percentile(a, q, axis=None, keepdims=False):
    """``reductions.percentile`` (reductions.py:644-658): ``np.percentile``
    (method 'linear', the reference passes no method)."""
    return np.percentile(a, q, axis=axis, keepdims=keepdims)


def quantile(a, q, axis=None, keepdims=False):
    """``reductions.quantile`` (reductions.py:806-820): ``np.quantile``."""
    return np.quantile(a, q, axis=axis, keepdims=keepdims)


def nanmedian(a, axis=None, keepdims=False):
    """``nan_ops.nanmedian`` (nan_ops.py:435-441): ``np.nanmedian``."""
    return np.nanmedian(a, axis=axis, keepdims=keepdims)


def nanpercentile(a, q, axis=None, keepdims=False):
    """``nan_ops.nanpercentile`` (nan_ops.py:763-780): ``np.nanpercentile``."""
    return np.nanpercentile(a, q, axis=axis, keepdims=keepdims)


def nanquantile(a, q, axis=None, keepdims=False):
    """``nan_ops.nanquantile`` (nan_ops.py:783-800): ``np.nanquantile``."""
    return np.nanquantile(a, q, axis=axis, keepdims=keepdims)


def unique(a, return_index=False, return_inverse=False, return_counts=False, axis=None):
    """``sorting.unique`` (sorting.py:200-215): ``np.unique`` (equal_nan=True:
    NaNs merge into one value)."""
    return np.unique(a, return_index=return_index, return_inverse=return_inverse, return_counts=return_counts,
                     axis=axis)


def lexsort(keys):
    """``sorting.lexsort`` (sorting.py:274-278): ``np.lexsort`` (stable, the
    last key primary)."""
    return np.lexsort(keys)


# ---------------------------------------------------------------- distributed merge
# The reference is single-device; its full reductions (ndarray._reduce,
# ndarray.py:1895-1963; reductions.var, reductions.py:525-584;
# reductions.argmax, reductions.py:381-418) are what a block-distributed
# array must reproduce.  These two functions restate, in numpy, the per-shard
# partial that the GPU writes (mmp_reduce_partial) and the ordered merge that
# folds the gathered partials (mmp_merge_partials), so that the merge rule is
# checked on CPU (gloo ranks) and the GPU merge kernel against this.

PARTIAL_FIELDS = ("s1", "s2", "shift", "count", "ival", "index")


def shard_partial(op, x, index_base=0):
    """The partial of one shard: a dict with the fields of ``mmp_partial``.
    Sums are float64 (floats) or exact int64 (integers); var keeps the shifted
    moments around the shard's first element; argmax/argmin keep (value,
    global index), numpy's first occurrence with NaN first."""
    x = np.asarray(x).reshape(-1)
    p = dict(s1=0.0, s2=0.0, shift=0.0, count=0, ival=0, index=-1)
    isf = x.dtype.kind == "f"
    n = x.size
    if op in ("sum", "mean"):
        p["count"] = n
        if isf:
            p["s1"] = float(x.astype(np.float64).sum())
        else:
            p["ival"] = int(x.astype(np.int64).sum())
            p["s1"] = float(p["ival"])
    elif op in ("var", "std"):
        p["count"] = n
        if n:
            k = float(x[0])
            d = x.astype(np.float64) - k
            p.update(s1=float(d.sum()), s2=float((d * d).sum()), shift=k)
    elif op in ("nansum", "nanmean"):
        ok = ~np.isnan(x)
        p.update(s1=float(x[ok].astype(np.float64).sum()), count=int(ok.sum()))
    elif op in ("nanvar", "nanstd"):
        v = x[~np.isnan(x)].astype(np.float64)
        if v.size:
            d = v - v[0]
            p.update(s1=float(d.sum()), s2=float((d * d).sum()), shift=float(v[0]), count=int(v.size))
    elif op in ("max", "min"):
        if n:
            v = (np.max if op == "max" else np.min)(x)
            p.update(s1=float(v), ival=0 if isf else int(v), count=n)
    elif op in ("argmax", "argmin"):
        p["count"] = n
        if n:
            i = int(np.argmax(x) if op == "argmax" else np.argmin(x))
            p.update(s1=float(x[i]), ival=0 if isf else int(x[i]), index=index_base + i)
    else:
        raise ValueError(op)
    return p


def merge_partials(op, parts, isfloat=True, ddof=0.0):
    """Fold shard partials in rank order into the reduction's result (the
    restatement of mmp_merge_partials).  var/std: each shard's shifted sums
    move to the first present shard's shift k_a with d = k_b - k_a,
    S1 += S1_b + n_b d, S2 += S2_b + d (2 S1_b + n_b d); then
    var = (S2 - S1^2/n) / (n - ddof)."""
    n = sum(int(p["count"]) for p in parts)
    if op in ("sum", "mean"):
        if isfloat:
            t = 0.0
            for p in parts:
                t += p["s1"]
        else:
            t = 0
            for p in parts:
                t += int(p["ival"])
        return t if op == "sum" else (float(t) / n if n else float("nan"))
    if op in ("nansum", "nanmean"):
        t = 0.0
        for p in parts:
            t += p["s1"]
        return t if op == "nansum" else (t / n if n else float("nan"))
    if op in ("var", "std", "nanvar", "nanstd"):
        s1 = s2 = k = 0.0
        seen = False
        for p in parts:
            if p["count"] <= 0:
                continue
            if not seen:
                s1, s2, k, seen = p["s1"], p["s2"], p["shift"], True
            else:
                nb, d = float(p["count"]), p["shift"] - k
                s2 += p["s2"] + d * (2.0 * p["s1"] + nb * d)
                s1 += p["s1"] + nb * d
        m2 = max(s2 - s1 * s1 / n, 0.0) if n else float("nan")
        dof = n - ddof
        if op.startswith("nan") and dof <= 0:
            return float("nan")
        var = m2 / max(dof, 0) if dof > 0 else (float("inf") if m2 > 0 else float("nan"))
        return float(np.sqrt(var)) if op.endswith("std") else var
    if op in ("max", "min"):
        best = None
        for p in parts:
            if p["count"] <= 0:
                continue
            v = p["s1"] if isfloat else p["ival"]
            if best is None:
                best = v
            elif isfloat and np.isnan(best):
                continue  # NaN propagates: the first NaN stays
            elif (isfloat and np.isnan(v)) or ((v > best) if op == "max" else (v < best)):
                best = v
        return best
    if op in ("argmax", "argmin"):
        best = None
        for p in parts:
            if p["index"] < 0:
                continue
            v, i = (p["s1"] if isfloat else p["ival"]), int(p["index"])
            if best is None:
                best = (v, i)
                continue
            bv, bi = best
            vn, bn = isfloat and np.isnan(v), isfloat and np.isnan(bv)
            if vn or bn:
                take = (i < bi) if (vn and bn) else vn
            elif v != bv:
                take = (v > bv) if op == "argmax" else (v < bv)
            else:
                take = i < bi
            if take:
                best = (v, i)
        return -1 if best is None else best[1]
    raise ValueError(op)
