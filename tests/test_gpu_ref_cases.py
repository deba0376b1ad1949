"""Cases of the reference's own test suite, restated against this build
through the drop-in name ``import macmetalpy``.

* RawKernel: the assertions of the reference's ``tests/test_rawkernel.py``
  (dtypes, 1-3 element grids, the 4-tuple error, a source that already has
  a ``_sync`` function, eight buffers, reuse, two kernels, a large grid)
  with the Metal sources rewritten as CUDA C (each kernel bounds-checks its
  thread index: a grid is a thread count rounded up to whole blocks);
* ``MetalBackend`` under the reference's name (``tests/test_synchronize.py``);
* range / differences / weighted mean / rounding / copy / expand_dims
  (``tests/test_reductions.py:528-697``, ``tests/test_math_ops.py``
  ``TestAround``/``TestCopy``, ``tests/test_ndarray.py`` ``TestExpandDims``);
* comparisons of a 0-d result with a Python bool
  (``tests/test_ndarray.py:916-945``), the error messages the reference's
  tests match (``tests/test_error_handling.py:100-105,256-266``), argmax
  ties (``tests/test_reductions.py:330-341``) and the 1M-element sum / add
  (``tests/test_edge_shapes.py:352-391``).

Tolerances are the reference conftest's (``tol_for``), exact for integers.
"""

import numpy as np
import numpy.testing as npt
import pytest

from conftest import tol_for

pytestmark = pytest.mark.gpu

NUMERIC = [np.float16, np.float32, np.int16, np.int32, np.int64, np.uint16, np.uint32, np.uint64]


@pytest.fixture(scope="module")
def mp():
    import macmetalpy
    return macmetalpy


def _arg(shape, dtype):
    """Deterministic small integers in the dtype (the reference's make_arg)."""
    n = int(np.prod(shape)) if shape else 1
    return (np.arange(1, n + 1) % 7 + 1).astype(dtype).reshape(shape)


def _eq(got, want, dtype):
    npt.assert_allclose(got.get() if hasattr(got, "get") else np.asarray(got), want, **tol_for(dtype))


# ---------------------------------------------------------------- RawKernel

DBL = {
    np.float32: ('extern "C" __global__ void dbl(const float* a, float* o, long long n) {'
                 ' long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; if (i < n) o[i] = a[i] * 2.0f; }',
                 "dbl"),
    np.int32: ('extern "C" __global__ void dbl_int(const int* a, int* o, long long n) {'
               ' long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; if (i < n) o[i] = a[i] * 2; }',
               "dbl_int"),
    np.float16: ('#include <cuda_fp16.h>\nextern "C" __global__ void dbl_half(const __half* a, __half* o, long long n) {'
                 ' long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;'
                 ' if (i < n) o[i] = __hmul(a[i], __float2half(2.0f)); }', "dbl_half"),
    np.uint32: ('extern "C" __global__ void dbl_uint(const unsigned* a, unsigned* o, long long n) {'
                ' long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; if (i < n) o[i] = a[i] * 2u; }',
                "dbl_uint"),
}
ADD = ('extern "C" __global__ void add_k(const float* a, const float* b, float* o, long long n) {'
       ' long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; if (i < n) o[i] = a[i] + b[i]; }')
SUM8 = ('extern "C" __global__ void sum8(const float* a, const float* b, const float* c, const float* d,'
        ' const float* e, const float* f, const float* g, const float* h, float* o, long long n) {'
        ' long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;'
        ' if (i < n) o[i] = a[i] + b[i] + c[i] + d[i] + e[i] + f[i] + g[i] + h[i]; }')
WITH_SYNC = DBL[np.float32][0].replace("void dbl(", "void dbl_sync(") + '\nextern "C" __global__ void _sync() {}'


@pytest.mark.parametrize("dtype", [np.float32, np.int32, np.float16, np.uint32])
def test_rawkernel_dtypes(mp, dtype):
    src, name = DBL[dtype]
    k = mp.RawKernel(src, name)
    a = mp.array([1, 2, 3], dtype=dtype)
    out = mp.empty(3, dtype=dtype)
    k(3, (a, out, 3))
    npt.assert_allclose(out.get(), [2, 4, 6], rtol=1e-2 if dtype == np.float16 else 0)


@pytest.mark.parametrize("grid", [4, (4,), (4, 1), (4, 1, 1)])
def test_rawkernel_grids(mp, grid):
    k = mp.RawKernel(*DBL[np.float32])
    a = mp.array([1, 2, 3, 4], dtype=np.float32)
    out = mp.empty(4, dtype=np.float32)
    k(grid, (a, out, 4))
    npt.assert_allclose(out.get(), [2, 4, 6, 8])


def test_rawkernel_4_tuple_raises(mp):
    k = mp.RawKernel(*DBL[np.float32])
    a = mp.array([1], dtype=np.float32)
    out = mp.empty(1, dtype=np.float32)
    with pytest.raises(ValueError, match="1-3"):
        k((1, 1, 1, 1), (a, out, 1))


def test_rawkernel_source_with_sync_function(mp):
    k = mp.RawKernel(WITH_SYNC, "dbl_sync")
    a = mp.array([10, 20], dtype=np.float32)
    out = mp.empty(2, dtype=np.float32)
    k(2, (a, out, 2))
    npt.assert_allclose(out.get(), [20, 40])


def test_rawkernel_eight_buffers_reuse_and_two_kernels(mp):
    k8 = mp.RawKernel(SUM8, "sum8")
    bufs = [mp.array([float(i + 1)], dtype=np.float32) for i in range(8)]
    out = mp.empty(1, dtype=np.float32)
    k8(1, (*bufs, out, 1))
    npt.assert_allclose(out.get(), [36.0])
    k1 = mp.RawKernel(*DBL[np.float32])
    for val in (1, 5, 10):
        a = mp.array([val], dtype=np.float32)
        o = mp.empty(1, dtype=np.float32)
        k1(1, (a, o, 1))
        npt.assert_allclose(o.get(), [val * 2])
    k2 = mp.RawKernel(ADD, "add_k")
    a = mp.array([1, 2, 3], dtype=np.float32)
    b = mp.array([4, 5, 6], dtype=np.float32)
    o1, o2 = mp.empty(3, dtype=np.float32), mp.empty(3, dtype=np.float32)
    k1(3, (a, o1, 3))
    k2(3, (a, b, o2, 3))
    npt.assert_allclose(o1.get(), [2, 4, 6])
    npt.assert_allclose(o2.get(), [5, 7, 9])


def test_rawkernel_large_grid(mp):
    n = 100_000
    k = mp.RawKernel(*DBL[np.float32])
    a = mp.array(np.ones(n, dtype=np.float32))
    out = mp.empty(n, dtype=np.float32)
    k(n, (a, out, n))
    npt.assert_allclose(out.get(), np.full(n, 2.0))


# ---------------------------------------------------------------- MetalBackend name


def test_metal_backend_synchronize(mp):
    from macmetalpy._metal_backend import MetalBackend

    be = MetalBackend()
    assert be is MetalBackend()
    a = mp.array([1.0, 4.0, 9.0], dtype=np.float32)
    b = mp.sqrt(a)
    be.synchronize()
    be.synchronize()
    assert not be._has_pending
    npt.assert_allclose(b.get(), [1, 2, 3], rtol=1e-6)


# ---------------------------------------------------------------- ptp / diff / average / around


@pytest.mark.parametrize("dtype", NUMERIC)
@pytest.mark.parametrize("shape", [(5,), (2, 3), (3, 4, 2)])
def test_ptp_and_diff(mp, dtype, shape):
    a = _arg(shape, dtype)
    A = mp.array(a)
    _eq(mp.ptp(A), np.ptp(a), dtype)
    _eq(mp.ptp(A, axis=0), np.ptp(a, axis=0), dtype)
    _eq(mp.diff(A), np.diff(a), dtype)
    _eq(mp.diff(A, n=2), np.diff(a, n=2), dtype)
    _eq(mp.diff(A, axis=0), np.diff(a, axis=0), dtype)
    d = mp.diff(A, axis=-1)
    assert d.dtype == np.diff(a, axis=-1).dtype


def test_diff_prepend_append_and_bool(mp):
    a = np.array([1, 4, 9, 16], dtype=np.int32)
    A = mp.array(a)
    npt.assert_array_equal(mp.diff(A, prepend=0).get(), np.diff(a, prepend=0))
    npt.assert_array_equal(mp.diff(A, append=[25, 36]).get(), np.diff(a, append=[25, 36]))
    m = np.array([[1, 2], [3, 5]], dtype=np.float32)
    npt.assert_array_equal(mp.diff(mp.array(m), axis=0, prepend=0).get(), np.diff(m, axis=0, prepend=0))
    b = np.array([True, True, False, True])
    npt.assert_array_equal(mp.diff(mp.array(b)).get(), np.diff(b))


@pytest.mark.parametrize("dtype", [np.float16, np.float32, np.int32, np.int64, np.uint16])
def test_average(mp, dtype):
    a = _arg((3, 4), dtype)
    A = mp.array(a)
    _eq(mp.average(A), np.average(a), dtype)
    _eq(mp.average(A, axis=0), np.average(a, axis=0), dtype)
    w = np.array([4, 3, 2, 1], dtype=dtype)
    got = mp.average(A, axis=1, weights=mp.array(w))
    want = np.average(a, axis=1, weights=w)
    assert got.dtype == want.dtype
    _eq(got, want, want.dtype)
    a1 = np.array([1, 2, 3, 4], dtype=dtype)
    got, scl = mp.average(mp.array(a1), weights=mp.array(w), returned=True)
    want, wscl = np.average(a1, weights=w, returned=True)
    _eq(got, want, np.asarray(want).dtype)
    _eq(scl, wscl, np.asarray(wscl).dtype)


@pytest.mark.parametrize("dtype", [np.float16, np.float32, np.int32, np.int64])
@pytest.mark.parametrize("decimals", [0, 2, -1])
def test_around(mp, dtype, decimals):
    rng = np.random.default_rng(decimals + 5)
    a = (rng.standard_normal(1000) * 300).astype(dtype)
    got = mp.around(mp.array(a), decimals)
    want = np.around(a, decimals)
    assert got.dtype == want.dtype
    npt.assert_array_equal(got.get(), want)
    npt.assert_array_equal(mp.round_(mp.array(a), decimals).get(), want)


def test_copy_and_expand_dims(mp):
    a = _arg((2, 3), np.float32)
    A = mp.array(a)
    C = mp.copy(A)
    C[0, 0] = 100
    assert float(A[0, 0].get()) == a[0, 0]
    for ax in (0, 1, 2, -1, (0, 2)):
        E = mp.expand_dims(A, ax)
        assert E.shape == np.expand_dims(a, ax).shape
        npt.assert_array_equal(E.get(), np.expand_dims(a, ax))


# ---------------------------------------------------------------- semantics the reference tests pin


def test_zero_d_result_against_python_bool(mp):
    z = mp.array(np.zeros((3, 4), dtype=np.float32))
    o = mp.array(np.ones((3, 4), dtype=np.float32))
    assert z.any() == False  # noqa: E712  (the reference test's own form)
    assert o.all() == True  # noqa: E712
    assert (mp.array(np.array([1, 0, 2], np.int32)) != False).get().tolist() == [True, False, True]  # noqa: E712


def test_error_messages(mp):
    with pytest.raises(ValueError, match="shape mismatch"):
        mp.zeros((2, 3), dtype=mp.float32) @ mp.zeros((4, 5), dtype=mp.float32)
    # batched @ (numpy semantics): the one deliberate divergence from
    # test_error_handling.py:116-121, which expects ValueError
    c = mp.ones((2, 3, 4), dtype=mp.float32) @ mp.ones((4, 5), dtype=mp.float32)
    assert c.shape == (2, 3, 5) and float(c.get()[1, 2, 4]) == 4.0
    with pytest.raises(TypeError, match="size-1"):
        float(mp.arange(5, dtype=mp.float32))
    with pytest.raises(TypeError, match="size-1"):
        int(mp.arange(5, dtype=mp.int32))
    assert float(mp.array([2.5], dtype=mp.float32)) == 2.5


@pytest.mark.parametrize("dtype", NUMERIC)
def test_argmax_ties_first_index(mp, dtype):
    a = np.array([3, 3, 1, 2], dtype=dtype)
    assert int(mp.argmax(mp.array(a))) == int(np.argmax(a)) == 0
    e = np.array([5, 5, 5], dtype=dtype)
    assert int(mp.argmax(mp.array(e))) == 0
    assert int(mp.argmin(mp.array(e))) == 0


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_large_sum_and_add(mp, dtype):
    n = 1_000_000
    a = mp.ones(n, dtype=dtype)
    s = mp.sum(a)
    if dtype == np.float32:
        npt.assert_allclose(float(s.get()), float(n), rtol=1e-4)
    else:
        s.get()
    r = (a + a).get()
    assert r.shape == (n,) and r[0] == 2 and r[-1] == 2
