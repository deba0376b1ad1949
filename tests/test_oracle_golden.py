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
