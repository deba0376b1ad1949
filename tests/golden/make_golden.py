"""Generate the golden vectors in ``golden_v1.npz`` from the REFERENCE itself.

Run in a container that has the reference checked out (read-only); its
path is the first argument or ``$MMP_REFERENCE`` (required: there is no
default); the GPU box never runs this.
The reference refuses to import off macOS (``src/macmetalpy/__init__.py:5-6``)
and its Metal path cannot run on Linux, so the script sets
``sys.platform = "darwin"`` only while importing, then raises every CPU/GPU
size threshold (``ndarray.py:41-44`` and the per-op tables ``:113-132``,
``reductions.py:378``) so that each op takes the reference's own CPU branch
-- the path the B200 build must match.  Paths whose only large-size branch is
Metal are not exercised here (sizes stay below ``nan_ops``/``matmul``'s
literal 4,194,304 thresholds), except ``__matmul__``, which has no CPU
branch: for it the script records ``np.matmul``, the function the
reference's ``cp.matmul`` CPU branch calls (``linalg_top.py:99-102``).

Every input is seeded (numpy ``default_rng``) and shaped like the BASELINE
configs at reduced size.  Usage:
``python tests/golden/make_golden.py <reference checkout>``.
"""

from __future__ import annotations

import os
import sys
import warnings

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MMP_REFERENCE", "")


def import_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "src", "macmetalpy")):
        raise SystemExit("pass the reference checkout as the first argument or in $MMP_REFERENCE")
    sys.path.insert(0, os.path.join(REF, "src"))
    saved = sys.platform
    sys.platform = "darwin"
    try:
        import macmetalpy as mp
    finally:
        sys.platform = saved
    nd = sys.modules["macmetalpy.ndarray"]
    big = 1 << 62
    for name in ("_GPU_THRESHOLD", "_GPU_THRESHOLD_LIGHT", "_GPU_THRESHOLD_MEMORY", "_GPU_REDUCTION_THRESHOLD"):
        setattr(nd, name, big)
    for table in (nd._UNARY_THRESHOLD, nd._BINARY_THRESHOLD):
        for k in table:
            table[k] = big
    sys.modules["macmetalpy.reductions"]._GPU_THRESHOLD_MEMORY = big
    return mp


def main():
    mp = import_reference()
    warnings.simplefilter("ignore")
    g = {}
    # C1: fused elementwise + reduction, reduced from 2^20 to 4096 elements
    rng = np.random.default_rng(0)
    x = rng.standard_normal(4096).astype(np.float32)
    X = mp.array(x)
    y = mp.sqrt(mp.abs(X)) + mp.exp(-X ** 2)
    g["c1_x"] = x
    g["c1_y"] = y.get()
    g["c1_sum"] = np.asarray(mp.sum(y).get())
    g["c1_mean"] = np.asarray(mp.mean(y).get())

    # C2: binary ufuncs (float32, int32) and a broadcast add
    rng = np.random.default_rng(1)
    n = 4096
    a = rng.uniform(-1000, 1000, n).astype(np.float32)
    b = (rng.uniform(1, 50, n) * rng.choice([-1, 1], n)).astype(np.float32)
    ai = rng.integers(-1000, 1000, n).astype(np.int32)
    bi = (rng.integers(1, 50, n) * rng.choice([-1, 1], n)).astype(np.int32)
    A, B, AI, BI = mp.array(a), mp.array(b), mp.array(ai), mp.array(bi)
    g["c2_a"], g["c2_b"], g["c2_ai"], g["c2_bi"] = a, b, ai, bi
    g["c2_add_f32"] = mp.add(A, B).get()
    g["c2_floordiv_f32"] = mp.floor_divide(A, B).get()
    g["c2_mod_f32"] = (A % B).get()
    g["c2_logaddexp_f32"] = mp.logaddexp(A, B).get()
    g["c2_add_i32"] = mp.add(AI, BI).get()
    g["c2_floordiv_i32"] = mp.floor_divide(AI, BI).get()
    g["c2_mod_i32"] = (AI % BI).get()
    r = rng.standard_normal((64, 1)).astype(np.float32)
    c = rng.standard_normal((1, 128)).astype(np.float32)
    g["c2_bc_r"], g["c2_bc_c"] = r, c
    g["c2_bc_add"] = (mp.array(r) + mp.array(c)).get()
    # edge operands: signed zeros, exact multiples, infinities, NaN
    ea = np.array([0.0, -0.0, 7.0, -7.0, 7.5, -7.5, np.inf, -np.inf, np.nan, 1e30, -1e-30, 5.0],
                  np.float32)
    eb = np.array([3.0, 3.0, -3.5, 3.5, 2.5, 2.5, 2.0, 2.0, 1.0, 3.0, 7.0, np.inf], np.float32)
    g["c2_edge_a"], g["c2_edge_b"] = ea, eb
    g["c2_edge_floordiv"] = mp.floor_divide(mp.array(ea), mp.array(eb)).get()
    g["c2_edge_mod"] = (mp.array(ea) % mp.array(eb)).get()
    g["c2_edge_logaddexp"] = mp.logaddexp(mp.array(ea), mp.array(eb)).get()
    ia = np.array([7, -7, 7, -7, 0, -2147483648, 2147483647, 5], np.int32)
    ib = np.array([2, 2, -2, -2, 5, -1, 1, 0], np.int32)
    g["c2_iedge_a"], g["c2_iedge_b"] = ia, ib
    g["c2_iedge_floordiv"] = mp.floor_divide(mp.array(ia), mp.array(ib)).get()
    g["c2_iedge_mod"] = (mp.array(ia) % mp.array(ib)).get()

    # C3: reductions on a (64, 96) matrix
    rng = np.random.default_rng(2)
    M = rng.standard_normal((64, 96)).astype(np.float32)
    MI = rng.integers(-100, 101, (64, 96)).astype(np.int32)
    MN = M.copy()
    nan_idx = rng.choice(M.size, M.size // 100, replace=False)
    MN.reshape(-1)[nan_idx] = np.nan
    g["c3_m"], g["c3_mi"], g["c3_mn"] = M, MI, MN
    Md, MId, MNd = mp.array(M), mp.array(MI), mp.array(MN)
    for nm, fn in (("sum", mp.sum), ("mean", mp.mean), ("var", mp.var)):
        g[f"c3_{nm}"] = np.asarray(fn(Md).get())
        for ax in (0, 1):
            g[f"c3_{nm}_ax{ax}"] = fn(Md, axis=ax).get()
    g["c3_argmax"] = np.asarray(mp.argmax(Md))
    g["c3_argmax_ax0"] = mp.argmax(Md, axis=0).get()
    g["c3_argmax_ax1"] = mp.argmax(Md, axis=1).get()
    g["c3_isum"] = np.asarray(mp.sum(MId).get())
    g["c3_nansum"] = np.asarray(mp.nansum(MNd).get())
    g["c3_nanmean"] = np.asarray(mp.nanmean(MNd).get())
    tie = np.array([3, 7, 7, 1, 7], np.float32)
    g["c3_tie"], g["c3_tie_argmax"] = tie, np.asarray(mp.argmax(mp.array(tie)))

    # C4: scans
    rng = np.random.default_rng(3)
    si = rng.integers(-100, 101, 8192).astype(np.int32)
    sf = rng.uniform(0, 1, 8192).astype(np.float32)
    s2 = rng.standard_normal((16, 512)).astype(np.float32)
    g["c4_si"], g["c4_sf"], g["c4_s2"] = si, sf, s2
    g["c4_cumsum_i32"] = mp.cumsum(mp.array(si)).get()
    g["c4_cumsum_f32"] = mp.cumsum(mp.array(sf)).get()
    g["c4_cumsum_ax1"] = mp.cumsum(mp.array(s2), axis=1).get()

    # C5: matmul
    rng = np.random.default_rng(4)
    ma = (rng.standard_normal((64, 96)) / np.sqrt(96)).astype(np.float32)
    mb = (rng.standard_normal((96, 80)) / np.sqrt(96)).astype(np.float32)
    ba = (rng.standard_normal((4, 32, 48)) / np.sqrt(48)).astype(np.float32)
    bb = (rng.standard_normal((4, 48, 40)) / np.sqrt(48)).astype(np.float32)
    ha = (rng.standard_normal((64, 64)) / 8).astype(np.float16)
    hb = (rng.standard_normal((64, 64)) / 8).astype(np.float16)
    g["c5_a"], g["c5_b"], g["c5_ba"], g["c5_bb"], g["c5_ha"], g["c5_hb"] = ma, mb, ba, bb, ha, hb
    g["c5_mm"] = mp.matmul(mp.array(ma), mp.array(mb)).get()
    g["c5_bmm"] = mp.matmul(mp.array(ba), mp.array(bb)).get()
    g["c5_hmm"] = mp.matmul(mp.array(ha), mp.array(hb)).get()

    out = os.path.join(HERE, "golden_v1.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out}: {len(g)} arrays, {os.path.getsize(out)} bytes")
    logic_golden(mp)
    nan_golden(mp)
    sort_golden(mp)
    index_golden(mp)
    order_golden(mp)


def order_golden(mp):
    """median / percentile / quantile (``reductions.py:627-820``), their
    nan-versions (``nan_ops.py:435-800``, below the 4,194,304-element
    threshold: the CPU branch), unique with first indices, inverse and
    counts (``sorting.py:200-215``) and lexsort (``sorting.py:274-278``),
    called through the reference."""
    g = {}
    rng = np.random.default_rng(11)
    a = (rng.standard_normal((9, 37)) * 10).astype(np.float32)
    an = a.copy()
    an[rng.random(a.shape) < 0.2] = np.nan
    an[3] = np.nan
    ai = rng.integers(-50, 50, (9, 37)).astype(np.int32)
    u = rng.integers(-20, 20, 600).astype(np.int32)
    uf = rng.standard_normal(800).astype(np.float32).round(1)
    uf[rng.random(800) < 0.05] = np.nan
    k1 = rng.integers(0, 5, 300).astype(np.int32)
    k2 = rng.standard_normal(300).astype(np.float32).round(0)
    g.update(a=a, an=an, ai=ai, u=u, uf=uf, k1=k1, k2=k2)
    A, AN, AI = mp.array(a), mp.array(an), mp.array(ai)
    for ax in (None, 0, 1):
        t = "n" if ax is None else str(ax)
        g[f"median_{t}"] = np.asarray(mp.median(A, axis=ax).get())
        g[f"median_i_{t}"] = np.asarray(mp.median(AI, axis=ax).get())
        g[f"pct37_{t}"] = np.asarray(mp.percentile(A, 37.5, axis=ax).get())
        g[f"pct_list_{t}"] = np.asarray(mp.percentile(A, [10, 50, 90], axis=ax).get())
        g[f"pct_i_{t}"] = np.asarray(mp.percentile(AI, 30, axis=ax).get())
        g[f"q03_{t}"] = np.asarray(mp.quantile(A, 0.3, axis=ax).get())
        g[f"nanmedian_{t}"] = np.asarray(mp.nanmedian(AN, axis=ax).get())
        g[f"nanpct_{t}"] = np.asarray(mp.nanpercentile(AN, 12.5, axis=ax).get())
        g[f"nanq_{t}"] = np.asarray(mp.nanquantile(AN, 0.6, axis=ax).get())
    for name, v in (("u", u), ("uf", uf)):
        vals, idx, inv, cnt = mp.unique(mp.array(v), return_index=True, return_inverse=True, return_counts=True)
        g[f"unique_{name}"] = vals.get()
        g[f"unique_{name}_index"] = idx.get()
        g[f"unique_{name}_inverse"] = inv.get()
        g[f"unique_{name}_counts"] = cnt.get()
    g["lexsort"] = mp.lexsort([mp.array(k1), mp.array(k2)]).get()
    out = os.path.join(HERE, "golden_order_v1.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out}: {len(g)} arrays, {os.path.getsize(out)} bytes")


def index_golden(mp):
    """Advanced indexing and the indexing routines through the reference's
    own __getitem__ / __setitem__ (numpy on the host, ``ndarray.py:874-957``)
    and ``indexing.py`` functions."""
    g = {}
    rng = np.random.default_rng(8)
    a = rng.standard_normal((6, 7, 8)).astype(np.float32)
    m = rng.standard_normal((6, 7, 8)).astype(np.float32) > 0.3
    i0 = np.array([5, 0, -1, 2, 2], np.int64)
    i1 = np.array([[1, 6], [0, -7]], np.int64)
    i2 = np.array([7, 0, 3], np.int64)
    v = rng.integers(-50, 50, 40).astype(np.int32)
    g.update(a=a, m=m, i0=i0, i1=i1, i2=i2, v=v)
    A = mp.array(a)
    g["get_mask"] = A[mp.array(m)].get()
    g["get_i0"] = A[mp.array(i0)].get()
    g["get_i0_i2"] = A[mp.array(i0[:3]), :, mp.array(i2)].get()            # non-adjacent: B first
    g["get_s_i1"] = A[1:5, mp.array(i1)].get()                              # adjacent, 2-D index
    g["get_int_arr"] = A[2, :, mp.array(i2)].get()                           # int + array, separated
    g["get_i1_i1"] = A[mp.array(i1 % 6), mp.array(i1 % 7)].get()
    g["get_mask_rows"] = A[mp.array(m[:, 0, 0])].get()
    g["get_newaxis"] = A[None, mp.array(i0), ::2].get()
    V = mp.array(v)
    g["get_v_neg"] = V[mp.array(np.array([-1, -40, 3, 39]))].get()
    # advanced __setitem__: the reference applies ``np_data[key] = value`` on
    # the host copy and uploads it with ``set`` (ndarray.py:948-957), which
    # needs Metal; the assignment itself is recorded here
    b = a.copy()
    b[m] = -1.0
    g["set_mask_scalar"] = b
    b = a.copy()
    b[i0[:3], 2] = np.arange(24, dtype=np.float32).reshape(3, 8)
    g["set_i0_row"] = b
    b = a.copy()
    b[:, np.array([6, 0]), 1] = 7.0
    g["set_cols"] = b
    g["take_v"] = mp.take(V, mp.array(np.array([0, 5, 39, -2]))).get()
    g["take_ax1"] = mp.take(A, mp.array(np.array([6, 0, 3])), axis=1).get()
    g["take_wrap"] = mp.take(V, mp.array(np.array([40, -41, 100])), mode="wrap").get()
    g["take_clip"] = mp.take(V, mp.array(np.array([40, -41, 100])), mode="clip").get()
    ta = rng.integers(0, 8, (6, 7, 3)).astype(np.int64)
    g["ta"] = ta
    g["take_along"] = mp.take_along_axis(A, mp.array(ta), axis=2).get()
    nz = mp.nonzero(mp.array(m))
    for k, x in enumerate(nz):
        g[f"nonzero_{k}"] = x.get()
    g["flatnonzero"] = mp.flatnonzero(mp.array(m)).get()
    g["argwhere"] = mp.argwhere(mp.array(m[0])).get()
    cond = rng.random(7) < 0.5
    g["cond"] = cond
    g["compress_ax1"] = mp.compress(mp.array(cond), A, axis=1).get()
    g["extract"] = mp.extract(mp.array(m), A).get()
    P = mp.array(v.copy())
    mp.put(P, mp.array(np.array([0, 3, 39])), mp.array(np.array([100, 200], np.int32)))
    g["put"] = P.get()
    P = mp.array(v.copy())
    mp.putmask(P, mp.array(v > 0), mp.array(np.array([7, 8, 9], np.int32)))
    g["putmask"] = P.get()
    out = os.path.join(HERE, "golden_index_v1.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out}: {len(g)} arrays, {os.path.getsize(out)} bytes")


def sort_golden(mp):
    """sort / argsort below the reference's 262,144-element GPU threshold
    (``sorting.py:30,48``), i.e. its CPU branch: np.sort / np.argsort with
    the default kind; argsort inputs have no ties (numpy's default kind
    leaves their order unspecified).  searchsorted has a CPU branch only
    with a sorter (``sorting.py:270-272``, np.searchsorted); without one it
    always runs its Metal binary search (``:228-268``), so those cases record
    np.searchsorted, the function its fallback calls."""
    g = {}
    rng = np.random.default_rng(7)
    f = rng.standard_normal(5000).astype(np.float32)
    f[:9] = [np.nan, -np.inf, np.inf, 0.0, -0.0, np.nan, 1e-45, -1e-45, 3e38]
    i = rng.integers(-1000, 1000, 5000).astype(np.int32)
    d = rng.standard_normal(3000)
    u = rng.permutation(4000).astype(np.float32) * np.float32(0.5) - np.float32(700)
    m = rng.standard_normal((37, 53)).astype(np.float32)
    h = rng.standard_normal(2000).astype(np.float16)
    g.update(f=f, i=i, d=d, u=u, m=m, h=h)
    F, I, D, U, M, H = (mp.array(v) for v in (f, i, d, u, m, h))
    g["sort_f"] = mp.sort(F).get()
    g["sort_i"] = mp.sort(I).get()
    g["sort_d"] = mp.sort(D).get()
    g["sort_h"] = mp.sort(H).get()
    g["sort_m_ax0"] = mp.sort(M, axis=0).get()
    g["sort_m_ax1"] = mp.sort(M, axis=1).get()
    g["sort_m_none"] = mp.sort(M, axis=None).get()
    g["argsort_u"] = mp.argsort(U).get()
    g["argsort_m_ax0"] = mp.argsort(M, axis=0).get()
    g["argsort_m_ax1"] = mp.argsort(M, axis=1).get()
    sf = np.sort(f)
    q = np.concatenate([rng.standard_normal(500).astype(np.float32), f[:9], sf[100:110]])
    g["q"] = q
    Q = mp.array(q)
    g["ss_left"] = np.searchsorted(sf, q)
    g["ss_right"] = np.searchsorted(sf, q, side="right")
    si = np.sort(i)
    qi = rng.integers(-1100, 1100, 300).astype(np.int32)
    g["qi"] = qi
    g["ss_i_left"] = np.searchsorted(si, qi)
    g["ss_i_right"] = np.searchsorted(si, qi, side="right")
    perm = rng.permutation(5000)
    srt = np.argsort(f[perm[:4000]], kind="stable")
    g["perm_f"] = f[perm[:4000]]
    g["sorter"] = srt
    g["ss_sorter"] = mp.searchsorted(mp.array(f[perm[:4000]]), Q, sorter=mp.array(srt)).get()
    out = os.path.join(HERE, "golden_sort_v1.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out}: {len(g)} arrays, {os.path.getsize(out)} bytes")


def nan_golden(mp):
    """The remaining NaN-aware reductions and scans (``nan_ops.py:171-612``)
    on small float32 / int32 inputs with ~10% NaN, one all-NaN row and one
    all-NaN column; every call takes the reference's CPU branch."""
    g = {}
    rng = np.random.default_rng(6)
    m = rng.standard_normal((24, 40)).astype(np.float32)
    m[rng.random(m.shape) < 0.1] = np.nan
    m[5, :] = np.nan
    m[:, 7] = np.nan
    p = rng.uniform(0.9, 1.1, (24, 40)).astype(np.float32)
    p[rng.random(p.shape) < 0.1] = np.nan
    v = rng.standard_normal(1000).astype(np.float32)
    v[rng.random(1000) < 0.1] = np.nan
    mi = rng.integers(-5, 6, (24, 40)).astype(np.int32)
    g.update(m=m, p=p, v=v, mi=mi)
    M, P, V, MI = mp.array(m), mp.array(p), mp.array(v), mp.array(mi)
    g["nanprod"] = np.asarray(mp.nanprod(P).get())
    g["nanprod_ax0"] = mp.nanprod(P, axis=0).get()
    g["nanprod_ax1"] = mp.nanprod(P, axis=1).get()
    g["nancumsum"] = mp.nancumsum(V).get()
    g["nancumsum_ax1"] = mp.nancumsum(M, axis=1).get()
    g["nancumprod_ax0"] = mp.nancumprod(P, axis=0).get()
    g["nancumsum_i"] = mp.nancumsum(MI).get()
    for ddof in (0, 1):
        g[f"nanvar_d{ddof}"] = np.asarray(mp.nanvar(M, ddof=ddof).get())
        g[f"nanvar_ax0_d{ddof}"] = mp.nanvar(M, axis=0, ddof=ddof).get()
        g[f"nanvar_ax1_d{ddof}"] = mp.nanvar(M, axis=1, ddof=ddof).get()
        g[f"nanstd_ax1_d{ddof}"] = mp.nanstd(M, axis=1, ddof=ddof).get()
    g["nanvar_i"] = np.asarray(mp.nanvar(MI).get())
    g["nanargmax"] = np.asarray(mp.nanargmax(V))
    g["nanargmin"] = np.asarray(mp.nanargmin(V))
    mm = np.where(np.isnan(m), np.float32(0), m)
    mm[3, ::2] = np.nan  # rows with NaN but no all-NaN slice
    g["mm"] = mm
    MM = mp.array(mm)
    g["nanargmax_ax1"] = mp.nanargmax(MM, axis=1).get()
    g["nanargmin_ax0"] = mp.nanargmin(MM, axis=0).get()
    g["nanargmax_i_ax0"] = mp.nanargmax(MI, axis=0).get()
    out = os.path.join(HERE, "golden_nan_v1.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out}: {len(g)} arrays, {os.path.getsize(out)} bytes")


def logic_golden(mp):
    """Comparison / logical / bitwise / predicate ops (the next row after the
    C1-C5 path) through the reference's own functions and operators; sizes
    stay below its 4,194,304 CPU threshold (``bitwise_ops.py:32``;
    ``logic_ops`` and ``math_ops.py:647`` use the same literal), so every
    call takes its CPU branch.  ``~`` of a bool array has no CPU branch
    (``ndarray.py:1687-1695`` runs the Metal ``bool_not_op``) and is not
    recorded."""
    g = {}
    rng = np.random.default_rng(5)
    fe = np.array([0.0, -0.0, 1.5, -2.5, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 3e38, 0.5, -0.5],
                  np.float32)
    f = np.concatenate([fe, rng.standard_normal(244).astype(np.float32)])
    f2 = f.copy()
    f2[::3] += np.float32(1e-6) * f2[::3]
    f2[5::7] = np.nan
    i = rng.integers(-1000, 1000, 256).astype(np.int32)
    i[:8] = [0, 1, -1, 2147483647, -2147483648, 7, -7, 12345]
    j = rng.integers(-40, 41, 256).astype(np.int32)
    j[:8] = [0, 1, 31, 32, 33, -1, 100, 5]
    bl = rng.random(256) < 0.5
    bl2 = rng.random(256) < 0.5
    w = rng.integers(-(1 << 40), 1 << 40, 64).astype(np.int64)
    w2 = rng.integers(-(1 << 40), 1 << 40, 64).astype(np.int64)
    g.update(f=f, f2=f2, i=i, j=j, bl=bl, bl2=bl2, w=w, w2=w2)
    F, F2, I, J, BL, BL2, W, W2 = (mp.array(v) for v in (f, f2, i, j, bl, bl2, w, w2))
    for nm in ("logical_and", "logical_or", "logical_xor"):
        fn = getattr(mp, nm)
        g[f"{nm}_ff"] = fn(F, F2).get()
        g[f"{nm}_ii"] = fn(I, J).get()
        g[f"{nm}_bb"] = fn(BL, BL2).get()
    g["logical_not_f"] = mp.logical_not(F).get()
    g["logical_not_i"] = mp.logical_not(I).get()
    for nm in ("isnan", "isinf", "isfinite", "signbit"):
        g[f"{nm}_f"] = getattr(mp, nm)(F).get()
    g["signbit_i"] = mp.signbit(I).get()
    g["isclose"] = mp.isclose(F, F2).get()
    g["isclose_nan"] = mp.isclose(F, F2, equal_nan=True).get()
    g["isclose_tol"] = mp.isclose(F, F2, rtol=1e-3, atol=1e-2).get()
    g["allclose"] = np.asarray(mp.allclose(F, F2))
    g["allclose_self_nan"] = np.asarray(mp.allclose(F, F, equal_nan=True))
    g["array_equal"] = np.asarray(mp.array_equal(F, F))
    g["array_equal_nan"] = np.asarray(mp.array_equal(F, F, equal_nan=True))
    g["array_equal_i"] = np.asarray(mp.array_equal(I, I))
    m2 = rng.integers(-2, 3, (16, 24)).astype(np.int32)
    g["cnz_m"] = m2
    g["cnz"] = np.asarray(mp.count_nonzero(mp.array(m2)))
    g["cnz_ax0"] = mp.count_nonzero(mp.array(m2), axis=0).get()
    g["cnz_ax1"] = mp.count_nonzero(mp.array(m2), axis=1).get()
    g["cnz_f"] = np.asarray(mp.count_nonzero(F))
    g["nan_to_num"] = mp.nan_to_num(F).get()
    g["nan_to_num_v"] = mp.nan_to_num(F, nan=-1.0, posinf=9.0, neginf=-9.0).get()
    for nm in ("bitwise_and", "bitwise_or", "bitwise_xor", "left_shift", "right_shift"):
        fn = getattr(mp, nm)
        g[f"{nm}_ii"] = fn(I, J).get()
        g[f"{nm}_ww"] = fn(W, W2 if not nm.endswith("shift") else mp.array(w2 % 40)).get()
        g[f"{nm}_bb"] = fn(BL, BL2).get()
    g["invert_i"] = mp.invert(I).get()
    g["invert_w"] = mp.invert(W).get()
    g["invert_b"] = mp.invert(BL).get()
    g["op_and_ii"] = (I & J).get()
    g["op_or_ii"] = (I | J).get()
    g["op_xor_ii"] = (I ^ J).get()
    g["op_and_bb"] = (BL & BL2).get()
    g["op_or_bb"] = (BL | BL2).get()
    g["op_xor_bb"] = (BL ^ BL2).get()
    g["op_and_ff"] = (F & F2).get()
    g["op_inv_i"] = (~I).get()
    g["op_lshift_ii"] = (I << J).get()
    g["op_rshift_ii"] = (I >> J).get()
    g["op_and_scalar"] = (I & 0xFF).get()
    g["op_rand_scalar"] = (0xF0 & I).get()
    out = os.path.join(HERE, "golden_logic_v1.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out}: {len(g)} arrays, {os.path.getsize(out)} bytes")


if __name__ == "__main__":
    main()
