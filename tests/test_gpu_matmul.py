"""matmul vs float64 numpy: float32 (3xTF32 tensor cores) within 1e-5
relative Frobenius error, float16 with float32 accumulation, batched and
1-D cases, odd shapes (CUDA-core path), error semantics."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cp():
    import macmetalpy_b200 as cp
    return cp


def frob(got, a, b):
    r = np.matmul(a.astype(np.float64), b.astype(np.float64))
    return np.linalg.norm(np.asarray(got, np.float64) - r) / max(np.linalg.norm(r), 1e-30)


@pytest.mark.parametrize("m,k,n", [(128, 128, 256), (256, 512, 256), (1000, 300, 700), (64, 96, 80), (1, 1, 1),
                                   (7, 13, 5), (130, 260, 390), (512, 2048, 512)])
def test_f32(cp, m, k, n):
    rng = np.random.default_rng(m + k + n)
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    got = (cp.array(a) @ cp.array(b)).get()
    assert got.dtype == np.float32 and got.shape == (m, n)
    assert frob(got, a, b) <= 1e-5


@pytest.mark.parametrize("m,k,n", [(128, 128, 256), (256, 512, 512), (96, 72, 40)])
def test_f16(cp, m, k, n):
    rng = np.random.default_rng(1)
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float16)
    b = (rng.standard_normal((k, n))).astype(np.float16)
    got = cp.matmul(cp.array(a), cp.array(b)).get()
    assert got.dtype == np.float16
    assert frob(got, a, b) <= 2e-3


# float16 on the tensor cores: row pitches that are multiples of 8 elements
# are read in place by TMA (B as an MN-major operand), with ragged M, N and
# K edges zero-filled; other pitches go through the K-major pre-pass.
@pytest.mark.parametrize("m,k,n", [(1000, 304, 712), (130, 264, 392), (2048, 2048, 2048), (256, 8, 1024),
                                   (1000, 300, 700), (129, 257, 255)])
def test_f16_tensor_core_paths(cp, m, k, n):
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float16)
    b = rng.standard_normal((k, n)).astype(np.float16)
    got = cp.matmul(cp.array(a), cp.array(b)).get()
    assert got.dtype == np.float16 and got.shape == (m, n)
    assert frob(got, a, b) <= 2e-3


def test_f16_batched_and_broadcast(cp):
    rng = np.random.default_rng(9)
    a = (rng.standard_normal((6, 256, 136)) / 12).astype(np.float16)
    b = rng.standard_normal((6, 136, 520)).astype(np.float16)
    got = cp.matmul(cp.array(a), cp.array(b)).get()
    assert got.shape == (6, 256, 520) and frob(got, a, b) <= 2e-3
    b2 = rng.standard_normal((136, 264)).astype(np.float16)
    got = cp.matmul(cp.array(a), cp.array(b2)).get()
    assert got.shape == (6, 256, 264) and frob(got, a, b2) <= 2e-3
    a2 = (rng.standard_normal((256, 136)) / 12).astype(np.float16)
    got = cp.matmul(cp.array(a2), cp.array(b)).get()
    assert got.shape == (6, 256, 520) and frob(got, a2, b) <= 2e-3


def test_batched_and_vectors(cp):
    rng = np.random.default_rng(2)
    a = (rng.standard_normal((8, 128, 64)) / 8).astype(np.float32)
    b = (rng.standard_normal((8, 64, 96)) / 8).astype(np.float32)
    got = cp.matmul(cp.array(a), cp.array(b)).get()
    assert got.shape == (8, 128, 96) and frob(got, a, b) <= 1e-5
    b2 = (rng.standard_normal((64, 96)) / 8).astype(np.float32)
    got = cp.matmul(cp.array(a), cp.array(b2)).get()
    assert frob(got, a, b2) <= 1e-5
    v = rng.standard_normal(64).astype(np.float32)
    np.testing.assert_allclose(cp.matmul(cp.array(a[0]), cp.array(v)).get(), a[0] @ v, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(float((cp.array(v) @ cp.array(v)).get()), float(v.astype(np.float64) @ v),
                               rtol=1e-5)
    ai = rng.integers(-5, 6, (33, 17)).astype(np.int32)
    bi = rng.integers(-5, 6, (17, 9)).astype(np.int32)
    np.testing.assert_array_equal(cp.matmul(cp.array(ai), cp.array(bi)).get(), ai @ bi)


def test_errors(cp):
    with pytest.raises(ValueError):
        cp.array(np.ones((3, 4), np.float32)) @ cp.array(np.ones((5, 6), np.float32))
    with pytest.raises(ValueError):
        cp.matmul(cp.array(np.float32(1)), cp.array(np.ones(3, np.float32)))
