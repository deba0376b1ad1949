"""Pin the CPU oracle to the reference: every oracle function reproduces the
golden vectors that tests/golden/make_golden.py recorded by running the
reference's own CPU path.  Exact equality everywhere (same inputs, same
numpy arithmetic), which is what makes the oracle a trustworthy checker."""

import os

import numpy as np
import pytest

from oracle import oracle as O

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_v1.npz"))


def eq(got, want):
    got, want = np.asarray(got), np.asarray(want)
    assert got.dtype == want.dtype, (got.dtype, want.dtype)
    assert got.shape == want.shape
    np.testing.assert_array_equal(got, want)


def test_c1():
    x = G["c1_x"]
    y = O.c1_expression(x)
    eq(y, G["c1_y"])
    eq(O.reduce_sum(y), G["c1_sum"])
    eq(O.reduce_mean(y), G["c1_mean"])


@pytest.mark.parametrize("suffix,a,b", [("f32", "c2_a", "c2_b"), ("i32", "c2_ai", "c2_bi")])
def test_c2_binary(suffix, a, b):
    a, b = G[a], G[b]
    eq(O.add(a, b), G[f"c2_add_{suffix}"])
    eq(O.floor_divide(a, b), G[f"c2_floordiv_{suffix}"])
    eq(O.mod(a, b), G[f"c2_mod_{suffix}"])
    if suffix == "f32":
        eq(O.logaddexp(a, b), G["c2_logaddexp_f32"])


def test_c2_mod_is_the_reference_composite_not_numpy_remainder():
    a, b = G["c2_a"], G["c2_b"]
    assert not np.array_equal(np.remainder(a, b), G["c2_mod_f32"])
    eq(O.mod(a, b), G["c2_mod_f32"])


def test_c2_edges_and_broadcast():
    eq(O.broadcast_add(G["c2_bc_r"], G["c2_bc_c"]), G["c2_bc_add"])
    ea, eb = G["c2_edge_a"], G["c2_edge_b"]
    eq(O.floor_divide(ea, eb), G["c2_edge_floordiv"])
    eq(O.mod(ea, eb), G["c2_edge_mod"])
    eq(O.logaddexp(ea, eb), G["c2_edge_logaddexp"])
    ia, ib = G["c2_iedge_a"], G["c2_iedge_b"]
    eq(O.floor_divide(ia, ib), G["c2_iedge_floordiv"])
    eq(O.mod(ia, ib), G["c2_iedge_mod"])


def test_c3_reductions():
    m = G["c3_m"]
    for nm, fn in (("sum", O.reduce_sum), ("mean", O.reduce_mean), ("var", O.reduce_var)):
        eq(fn(m), G[f"c3_{nm}"])
        for ax in (0, 1):
            eq(fn(m, axis=ax), G[f"c3_{nm}_ax{ax}"])
    assert O.argmax(m) == int(G["c3_argmax"])
    eq(O.argmax_axis(m, 0), G["c3_argmax_ax0"])
    eq(O.argmax_axis(m, 1), G["c3_argmax_ax1"])
    eq(O.reduce_sum(G["c3_mi"]), G["c3_isum"])
    eq(O.nansum(G["c3_mn"]), G["c3_nansum"])
    eq(O.nanmean(G["c3_mn"]), G["c3_nanmean"])
    assert O.argmax(G["c3_tie"]) == int(G["c3_tie_argmax"]) == 1


def test_c4_scans():
    eq(O.cumsum(G["c4_si"]), G["c4_cumsum_i32"])
    eq(O.cumsum(G["c4_sf"]), G["c4_cumsum_f32"])
    eq(O.cumsum(G["c4_s2"], axis=1), G["c4_cumsum_ax1"])


def test_c5_matmul():
    eq(O.matmul(G["c5_a"], G["c5_b"]), G["c5_mm"])
    eq(O.matmul(G["c5_ba"], G["c5_bb"]), G["c5_bmm"])
    eq(O.matmul(G["c5_ha"], G["c5_hb"]), G["c5_hmm"])


def test_resolve_dtype_rules():
    assert O.resolve_dtype(np.float64, "downcast") == np.float32
    assert O.resolve_dtype(np.float64, "cpu_fallback") == np.float64
    assert O.resolve_dtype(np.int8) == np.int16
    assert O.resolve_dtype(np.uint8) == np.uint16
    assert O.resolve_dtype(None) == np.float32


L = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_logic_v1.npz"))


def test_logic_predicates():
    f, f2, i, j, bl, bl2 = L["f"], L["f2"], L["i"], L["j"], L["bl"], L["bl2"]
    for nm in ("logical_and", "logical_or", "logical_xor"):
        eq(O.logical(nm, f, f2), L[f"{nm}_ff"])
        eq(O.logical(nm, i, j), L[f"{nm}_ii"])
        eq(O.logical(nm, bl, bl2), L[f"{nm}_bb"])
    eq(O.logical_not(f), L["logical_not_f"])
    eq(O.logical_not(i), L["logical_not_i"])
    for nm in ("isnan", "isinf", "isfinite", "signbit"):
        eq(O.predicate(nm, f), L[f"{nm}_f"])
    eq(O.predicate("signbit", i), L["signbit_i"])
    eq(O.isclose(f, f2), L["isclose"])
    eq(O.isclose(f, f2, equal_nan=True), L["isclose_nan"])
    eq(O.isclose(f, f2, rtol=1e-3, atol=1e-2), L["isclose_tol"])
    assert O.allclose(f, f2) == bool(L["allclose"])
    assert O.allclose(f, f, equal_nan=True) == bool(L["allclose_self_nan"])
    assert O.array_equal(f, f) == bool(L["array_equal"]) is False  # NaN != NaN
    assert O.array_equal(f, f, equal_nan=True) == bool(L["array_equal_nan"])
    assert O.array_equal(i, i) == bool(L["array_equal_i"])
    m = L["cnz_m"]
    assert O.count_nonzero(m) == int(L["cnz"])
    eq(O.count_nonzero(m, axis=0), L["cnz_ax0"])
    eq(O.count_nonzero(m, axis=1), L["cnz_ax1"])
    assert O.count_nonzero(f) == int(L["cnz_f"])
    eq(O.nan_to_num(f), L["nan_to_num"])
    eq(O.nan_to_num(f, nan=-1.0, posinf=9.0, neginf=-9.0), L["nan_to_num_v"])


def test_bitwise_and_operators():
    i, j, bl, bl2, w, w2, f, f2 = (L[k] for k in ("i", "j", "bl", "bl2", "w", "w2", "f", "f2"))
    for nm in ("bitwise_and", "bitwise_or", "bitwise_xor", "left_shift", "right_shift"):
        eq(O.bitwise(nm, i, j), L[f"{nm}_ii"])
        eq(O.bitwise(nm, w, w2 if not nm.endswith("shift") else w2 % 40), L[f"{nm}_ww"])
        eq(O.bitwise(nm, bl, bl2), L[f"{nm}_bb"])
    eq(O.invert(i), L["invert_i"])
    eq(O.invert(w), L["invert_w"])
    eq(O.invert(bl), L["invert_b"])
    eq(O.op_and(i, j), L["op_and_ii"])
    eq(O.op_or(i, j), L["op_or_ii"])
    eq(O.op_xor(i, j), L["op_xor_ii"])
    eq(O.op_and(bl, bl2), L["op_and_bb"])
    eq(O.op_or(bl, bl2), L["op_or_bb"])
    eq(O.op_xor(bl, bl2), L["op_xor_bb"])
    eq(O.op_and(f, f2), L["op_and_ff"])
    eq(O.op_invert(i), L["op_inv_i"])
    eq(O.op_shift("left_shift", i, j), L["op_lshift_ii"])
    eq(O.op_shift("right_shift", i, j), L["op_rshift_ii"])
    eq(O.op_and(i, 0xFF), L["op_and_scalar"])
    eq(O.bitwise("bitwise_and", 0xF0, i), L["op_rand_scalar"])


N = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_nan_v1.npz"))


def test_nan_reductions_and_scans():
    import warnings

    warnings.simplefilter("ignore", RuntimeWarning)
    m, p, v, mi, mm = N["m"], N["p"], N["v"], N["mi"], N["mm"]
    eq(O.nanprod(p), N["nanprod"])
    eq(O.nanprod(p, axis=0), N["nanprod_ax0"])
    eq(O.nanprod(p, axis=1), N["nanprod_ax1"])
    eq(O.nancumsum(v), N["nancumsum"])
    eq(O.nancumsum(m, axis=1), N["nancumsum_ax1"])
    eq(O.nancumprod(p, axis=0), N["nancumprod_ax0"])
    eq(O.nancumsum(mi), N["nancumsum_i"])
    for ddof in (0, 1):
        eq(O.nanvar(m, ddof=ddof), N[f"nanvar_d{ddof}"])
        eq(O.nanvar(m, axis=0, ddof=ddof), N[f"nanvar_ax0_d{ddof}"])
        eq(O.nanvar(m, axis=1, ddof=ddof), N[f"nanvar_ax1_d{ddof}"])
        eq(O.nanstd(m, axis=1, ddof=ddof), N[f"nanstd_ax1_d{ddof}"])
    eq(O.nanvar(mi), N["nanvar_i"])
    assert O.nanargmax(v) == int(N["nanargmax"])
    assert O.nanargmin(v) == int(N["nanargmin"])
    eq(O.nanargmax(mm, axis=1), N["nanargmax_ax1"])
    eq(O.nanargmin(mm, axis=0), N["nanargmin_ax0"])
    eq(O.nanargmax(mi, axis=0), N["nanargmax_i_ax0"])
    with pytest.raises(ValueError):
        O.nanargmax(m, axis=1)


S = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_sort_v1.npz"))


def test_sort_searchsorted():
    for k in ("f", "i", "d", "h"):
        eq(O.sort(S[k]), S[f"sort_{k}"])
    m = S["m"]
    eq(O.sort(m, axis=0), S["sort_m_ax0"])
    eq(O.sort(m, axis=1), S["sort_m_ax1"])
    eq(O.sort(m, axis=None), S["sort_m_none"])
    eq(O.argsort(S["u"]), S["argsort_u"])
    eq(O.argsort(m, axis=0), S["argsort_m_ax0"])
    eq(O.argsort(m, axis=1), S["argsort_m_ax1"])
    sf = np.sort(S["f"])
    eq(O.searchsorted(sf, S["q"]), S["ss_left"])
    eq(O.searchsorted(sf, S["q"], side="right"), S["ss_right"])
    si = np.sort(S["i"])
    eq(O.searchsorted(si, S["qi"]), S["ss_i_left"])
    eq(O.searchsorted(si, S["qi"], side="right"), S["ss_i_right"])
    eq(O.searchsorted(S["perm_f"], S["q"], sorter=S["sorter"]), S["ss_sorter"])


X = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_index_v1.npz"))


def test_advanced_indexing_and_routines():
    a, m, i0, i1, i2, v = (X[k] for k in ("a", "m", "i0", "i1", "i2", "v"))
    eq(O.getitem(a, m), X["get_mask"])
    eq(O.getitem(a, i0), X["get_i0"])
    eq(O.getitem(a, (i0[:3], slice(None), i2)), X["get_i0_i2"])
    eq(O.getitem(a, (slice(1, 5), i1)), X["get_s_i1"])
    eq(O.getitem(a, (2, slice(None), i2)), X["get_int_arr"])
    eq(O.getitem(a, (i1 % 6, i1 % 7)), X["get_i1_i1"])
    eq(O.getitem(a, m[:, 0, 0]), X["get_mask_rows"])
    eq(O.getitem(a, (None, i0, slice(None, None, 2))), X["get_newaxis"])
    eq(O.getitem(v, np.array([-1, -40, 3, 39])), X["get_v_neg"])
    eq(O.setitem(a, m, -1.0), X["set_mask_scalar"])
    eq(O.setitem(a, (i0[:3], 2), np.arange(24, dtype=np.float32).reshape(3, 8)), X["set_i0_row"])
    eq(O.setitem(a, (slice(None), np.array([6, 0]), 1), 7.0), X["set_cols"])
    eq(O.take(v, np.array([0, 5, 39, -2])), X["take_v"])
    eq(O.take(a, np.array([6, 0, 3]), axis=1), X["take_ax1"])
    eq(O.take(v, np.array([40, -41, 100]), mode="wrap"), X["take_wrap"])
    eq(O.take(v, np.array([40, -41, 100]), mode="clip"), X["take_clip"])
    eq(O.take_along_axis(a, X["ta"], 2), X["take_along"])
    for k, x in enumerate(O.nonzero(m)):
        eq(x, X[f"nonzero_{k}"])
    eq(O.flatnonzero(m), X["flatnonzero"])
    eq(O.argwhere(m[0]), X["argwhere"])
    eq(O.compress(X["cond"], a, axis=1), X["compress_ax1"])
    eq(O.extract(m, a), X["extract"])
    eq(O.put(v, np.array([0, 3, 39]), np.array([100, 200], np.int32)), X["put"])
    eq(O.putmask(v, v > 0, np.array([7, 8, 9], np.int32)), X["putmask"])


R = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_order_v1.npz"))


def test_order_statistics_unique_lexsort():
    a, an, ai = R["a"], R["an"], R["ai"]
    for ax in (None, 0, 1):
        t = "n" if ax is None else str(ax)
        eq(O.median(a, axis=ax), R[f"median_{t}"])
        eq(O.median(ai, axis=ax), R[f"median_i_{t}"])
        eq(O.percentile(a, 37.5, axis=ax), R[f"pct37_{t}"])
        eq(O.percentile(a, [10, 50, 90], axis=ax), R[f"pct_list_{t}"])
        eq(O.percentile(ai, 30, axis=ax), R[f"pct_i_{t}"])
        eq(O.quantile(a, 0.3, axis=ax), R[f"q03_{t}"])
        eq(O.nanmedian(an, axis=ax), R[f"nanmedian_{t}"])
        eq(O.nanpercentile(an, 12.5, axis=ax), R[f"nanpct_{t}"])
        eq(O.nanquantile(an, 0.6, axis=ax), R[f"nanq_{t}"])
    for name in ("u", "uf"):
        vals, idx, inv, cnt = O.unique(R[name], return_index=True, return_inverse=True, return_counts=True)
        eq(vals, R[f"unique_{name}"])
        eq(idx, R[f"unique_{name}_index"])
        eq(inv, R[f"unique_{name}_inverse"])
        eq(cnt, R[f"unique_{name}_counts"])
    eq(O.lexsort([R["k1"], R["k2"]]), R["lexsort"])
