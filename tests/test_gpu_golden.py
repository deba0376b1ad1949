"""GPU parity against the golden vectors recorded from the reference.

Bit-exact for integer ops, floor_divide and mod; float32 transcendental
results within 2 ulp of the float64-evaluated value; float reductions within
1e-4 relative error of the float64-accumulated result; float32 matmul
within 1e-5 relative Frobenius error."""

import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_v1.npz"))


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    return cp


def exact(got, want):
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.dtype == want.dtype, (got.dtype, want.dtype)
    np.testing.assert_array_equal(got, want)


def rel(got, ref64):
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref64)) / max(np.max(np.abs(ref64)), 1e-30))


def test_c1_expression_and_fused_reductions(cp):
    x = G["c1_x"]
    X = cp.array(x)
    y = cp.sqrt(cp.abs(X)) + cp.exp(-X ** 2)
    x64 = x.astype(np.float64)
    y64 = np.sqrt(np.abs(x64)) + np.exp(-(x64 * x64))
    assert O.ulp_error(y.get(), y64).max() <= 2.0
    # libm (reference) and CUDA exp may differ by an ulp: within 2 ulp of the reference
    assert (np.abs(y.get() - G["c1_y"]) <= 2 * np.spacing(G["c1_y"])).all()
    s = cp.sum(y)  # fused: the expression runs inside the reduction
    m = cp.mean(y)
    assert s.dtype == np.float32 and m.dtype == np.float32
    assert abs(float(s.get()) - y64.sum()) / y64.sum() <= 1e-4
    assert abs(float(m.get()) - y64.mean()) / y64.mean() <= 1e-4


@pytest.mark.parametrize("suffix,a,b", [("f32", "c2_a", "c2_b"), ("i32", "c2_ai", "c2_bi")])
def test_c2_binary_bit_exact(cp, suffix, a, b):
    A, B = cp.array(G[a]), cp.array(G[b])
    exact(cp.add(A, B).get(), G[f"c2_add_{suffix}"])
    exact(cp.floor_divide(A, B).get(), G[f"c2_floordiv_{suffix}"])
    exact((A % B).get(), G[f"c2_mod_{suffix}"])
    exact((A // B).get(), G[f"c2_floordiv_{suffix}"])
    exact(cp.mod(A, B).get(), G[f"c2_mod_{suffix}"])


def test_c2_logaddexp_ulp(cp):
    a, b = G["c2_a"], G["c2_b"]
    got = cp.logaddexp(cp.array(a), cp.array(b)).get()
    ref = np.logaddexp(a.astype(np.float64), b.astype(np.float64))
    assert O.ulp_error(got, ref).max() <= 2.0
    np.testing.assert_allclose(got, G["c2_logaddexp_f32"], rtol=3e-7)


def test_c2_edges(cp):
    ea, eb = cp.array(G["c2_edge_a"]), cp.array(G["c2_edge_b"])
    exact(cp.floor_divide(ea, eb).get(), G["c2_edge_floordiv"])
    exact((ea % eb).get(), G["c2_edge_mod"])
    got = cp.logaddexp(ea, eb).get()
    np.testing.assert_allclose(got, G["c2_edge_logaddexp"], rtol=3e-7)
    ia, ib = cp.array(G["c2_iedge_a"]), cp.array(G["c2_iedge_b"])
    exact(cp.floor_divide(ia, ib).get(), G["c2_iedge_floordiv"])
    exact((ia % ib).get(), G["c2_iedge_mod"])


def test_c2_broadcast_add(cp):
    exact((cp.array(G["c2_bc_r"]) + cp.array(G["c2_bc_c"])).get(), G["c2_bc_add"])


def test_c3_reductions(cp):
    m = G["c3_m"]
    M = cp.array(m)
    m64 = m.astype(np.float64)
    for nm, fn, ref in (("sum", cp.sum, np.sum), ("mean", cp.mean, np.mean), ("var", cp.var, np.var)):
        got = fn(M)
        assert got.dtype == G[f"c3_{nm}"].dtype
        assert rel(got.get(), ref(m64)) <= 1e-4, nm
        for ax in (0, 1):
            g = fn(M, axis=ax)
            assert g.dtype == G[f"c3_{nm}_ax{ax}"].dtype
            r64 = ref(m64, axis=ax)
            assert np.max(np.abs(g.get() - r64) / np.maximum(np.abs(r64), 1e-3)) <= 1e-4, (nm, ax)
    assert cp.argmax(M) == int(G["c3_argmax"])
    exact(cp.argmax(M, axis=0).get(), G["c3_argmax_ax0"])
    exact(cp.argmax(M, axis=1).get(), G["c3_argmax_ax1"])
    exact(cp.sum(cp.array(G["c3_mi"])).get(), G["c3_isum"])
    mn = G["c3_mn"]
    assert rel(cp.nansum(cp.array(mn)).get(), np.nansum(mn.astype(np.float64))) <= 1e-4
    assert rel(cp.nanmean(cp.array(mn)).get(), np.nanmean(mn.astype(np.float64))) <= 1e-4
    assert cp.argmax(cp.array(G["c3_tie"])) == 1


def test_c4_scans(cp):
    exact(cp.cumsum(cp.array(G["c4_si"])).get(), G["c4_cumsum_i32"])
    sf = G["c4_sf"]
    got = cp.cumsum(cp.array(sf)).get()
    assert got.dtype == np.float32
    assert rel(got, np.cumsum(sf.astype(np.float64))) <= 1e-4
    s2 = G["c4_s2"]
    g2 = cp.cumsum(cp.array(s2), axis=1).get()
    r2 = np.cumsum(s2.astype(np.float64), axis=1)
    assert np.max(np.abs(g2 - r2)) / np.max(np.abs(r2)) <= 1e-4


def test_c5_matmul(cp):
    def frob(got, a, b):
        r = np.matmul(a.astype(np.float64), b.astype(np.float64))
        return np.linalg.norm(np.asarray(got, np.float64) - r) / np.linalg.norm(r)

    a, b = G["c5_a"], G["c5_b"]
    got = cp.matmul(cp.array(a), cp.array(b)).get()
    assert got.dtype == np.float32 and frob(got, a, b) <= 1e-5
    ba, bb = G["c5_ba"], G["c5_bb"]
    got = cp.matmul(cp.array(ba), cp.array(bb)).get()
    assert got.shape == (4, 32, 40) and frob(got, ba, bb) <= 1e-5
    ha, hb = G["c5_ha"], G["c5_hb"]
    got = cp.matmul(cp.array(ha), cp.array(hb)).get()
    assert got.dtype == np.float16
    assert frob(got, ha, hb) <= 2e-3
    np.testing.assert_allclose(got.astype(np.float32), G["c5_hmm"].astype(np.float32), rtol=2e-2, atol=2e-3)
