"""API-level behaviour on the GPU: RawKernel (CUDA C source, thread-count
grids, 1-3-D, argument kinds), get/set/synchronize, creation, views,
device errors raise, no silent CPU path."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    return cp


SRC = r'''
extern "C" __global__ void axpy(const float* x, float* y, float a, long long n) {
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i < n) y[i] = a * x[i] + y[i];
}
extern "C" __global__ void fill2d(int* out, int w, int h) {
  int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
  if (x < w && y < h) out[y * w + x] = y * 1000 + x;
}
'''


def test_rawkernel(cp):
    n = 100003
    x = np.arange(n, dtype=np.float32)
    y = np.ones(n, np.float32)
    X, Y = cp.array(x), cp.array(y)
    k = cp.RawKernel(SRC, "axpy")
    k(n, (X, Y, np.float32(2.0), n))
    np.testing.assert_array_equal(Y.get(), 2 * x + 1)
    k2 = cp.RawKernel(SRC, "fill2d")
    O = cp.zeros((37, 53), dtype=np.int32)
    k2((53, 37), (O, 53, 37))
    yy, xx = np.mgrid[0:37, 0:53]
    np.testing.assert_array_equal(O.get(), yy * 1000 + xx)
    with pytest.raises(ValueError):
        k((1, 2, 3, 4), (X, Y, np.float32(1), n))


def test_rawkernel_compile_error(cp):
    with pytest.raises(RuntimeError):
        cp.RawKernel("extern \"C\" __global__ void bad( { }", "bad")(1, ())


def test_creation_and_transfer(cp):
    assert cp.zeros((3, 4)).dtype == np.float32
    np.testing.assert_array_equal(cp.ones((2, 2), dtype=np.int32).get(), np.ones((2, 2), np.int32))
    np.testing.assert_array_equal(cp.full((5,), 7.5).get(), np.full(5, 7.5, np.float32))
    np.testing.assert_array_equal(cp.arange(10).get(), np.arange(10))
    a = cp.empty((4, 4), dtype=np.float32)
    a.set(np.eye(4, dtype=np.float32))
    np.testing.assert_array_equal(a.get(), np.eye(4, dtype=np.float32))
    np.testing.assert_array_equal(cp.asnumpy(a), np.eye(4, dtype=np.float32))
    assert a.strides == (16, 4)
    cp.synchronize()


def test_reshape_transpose_views(cp):
    x = np.arange(60, dtype=np.int64).reshape(3, 4, 5)
    X = cp.array(x)
    np.testing.assert_array_equal(X.transpose(2, 0, 1).get(), x.transpose(2, 0, 1))
    np.testing.assert_array_equal(X.reshape(12, 5).get(), x.reshape(12, 5))
    np.testing.assert_array_equal(X.T.reshape(-1).get(), x.T.reshape(-1))
    np.testing.assert_array_equal(X[1:, ::2, -1].get(), x[1:, ::2, -1])
    np.testing.assert_array_equal(X[..., 1].get(), x[..., 1])
    np.testing.assert_array_equal(X.squeeze().get(), x)
    np.testing.assert_array_equal(X[:, None].get(), x[:, None])
    np.testing.assert_array_equal(X[[0, 2]].get(), x[[0, 2]])


def test_cuda_array_interface(cp):
    X = cp.array(np.arange(8, dtype=np.float32))
    cai = X.__cuda_array_interface__
    assert cai["shape"] == (8,) and cai["typestr"] == "<f4" and cai["data"][0] == X.data_ptr


def test_native_library_loaded(cp):
    import macmetalpy_b200._cuda_backend as cb
    assert cb.lib.mmp_abi_version() == 1
    assert cb.CudaBackend().sm_count > 0


def test_zero_d_arrays_keep_their_shape():
    import macmetalpy_b200 as cp
    for v in (3.5, np.float32(2.0), np.array(7, np.int32)):
        a = cp.array(v)
        assert a.shape == () and a.get().shape == ()
        assert float(a.get()) == float(v)
    b = cp.array(np.float32(1.0))
    b.set(np.float32(4.0))
    assert b.shape == () and float(b.get()) == 4.0


def test_streams_async_copies_and_pinned_memory():
    import macmetalpy_b200 as cp
    from macmetalpy_b200.cuda import Event, Stream, empty_pinned
    n = 1 << 22
    rng = np.random.default_rng(0)
    s_in, s_out = Stream(), Stream()
    src = empty_pinned((n,), np.float32)
    src[...] = rng.standard_normal(n).astype(np.float32)
    dst = empty_pinned((n,), np.float32)
    X = cp.empty((n,), dtype=np.float32)
    Y = cp.empty((n,), dtype=np.float32)
    for rep in range(3):  # uploads on a side stream, kernel on the library stream, download on another
        src[:8] = rep
        X.set(src, stream=s_in)
        cp.multiply(X, 2.0, out=Y)
        Y.get(stream=s_out, out=dst)
        s_out.synchronize()
        np.testing.assert_array_equal(dst, src * np.float32(2))
    e0, e1 = Event().record(), Event()
    cp.add(X, X, out=Y)
    e1.record()
    e1.synchronize()
    assert e0.elapsed_time(e1) >= 0.0
    with pytest.raises(ValueError):
        X.set(np.zeros(n + 1, np.float32), stream=s_in)
    v = dst[10:20]  # a view keeps the pinned block alive
    del dst
    assert v.shape == (10,)
