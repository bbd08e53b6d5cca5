"""GPU runs of traced plain kernels (tests/kernel_zoo.py) against NumPy:
the surface the reference's tests/test_thork.py covers — pointer loads and
stores, scalar and vector attributes, by-value constants, locals, loops,
shared memory, math intrinsics, atomics, warp reductions, device functions
and control flow — compiled through NVRTC for sm_100a."""

import numpy as np
import pytest

import thork_b200 as tk

import kernel_zoo

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def zoo():
    return kernel_zoo.build(tk)


def test_vec_add_bit_exact(zoo):
    rng = np.random.default_rng(0)
    a = rng.standard_normal(1 << 16, dtype=np.float32)
    b = rng.standard_normal(1 << 16, dtype=np.float32)
    out = np.zeros_like(a)
    zoo["vec_add"][(a.size // 256, 1, 1), (256, 1, 1)](out, a, b)
    np.testing.assert_array_equal(out, a + b)


def test_saxpy_grid_stride_with_constants(zoo):
    rng = np.random.default_rng(1)
    n = 10_000
    x = rng.standard_normal(n, dtype=np.float32)
    y = rng.standard_normal(n, dtype=np.float32)
    expected = y + np.float32(3) * x
    zoo["saxpy_strided"][(8, 1, 1), (128, 1, 1)](y, x, 3, n)
    np.testing.assert_allclose(y, expected, rtol=1e-6, atol=1e-6)


def test_row_dot_matmul(zoo):
    rng = np.random.default_rng(2)
    m = n = k = 128
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    c = np.zeros((m, n), np.float32)
    zoo["row_dot"][(n // 16, m // 16, 1), (16, 16, 1)](c, a, b, k, n)
    np.testing.assert_allclose(c, a @ b, atol=1e-3, rtol=1e-3)


def test_shared_tiled_matmul(zoo):
    rng = np.random.default_rng(3)
    m, n, k = 128, 64, 96
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    c = np.zeros((m, n), np.float32)
    zoo["tiled_mm"][(n // 16, m // 16, 1), (16, 16, 1)](c, a, b, m, n, k)
    np.testing.assert_allclose(c, a @ b, atol=1e-3, rtol=1e-3)


def test_math_intrinsics(zoo):
    rng = np.random.default_rng(4)
    a = rng.standard_normal(4096).astype(np.float32)
    out = np.zeros_like(a)
    zoo["softplus"][(32, 1, 1), (128, 1, 1)](out, a)
    np.testing.assert_allclose(out, np.log1p(np.exp(a)), atol=1e-5, rtol=1e-5)


def test_atomic_histogram_exact(zoo):
    rng = np.random.default_rng(5)
    values = rng.integers(0, 64, size=4096).astype(np.uint32)
    counts = np.zeros(16, np.uint32)
    zoo["bincount"][(32, 1, 1), (128, 1, 1)](counts, values, 16)
    np.testing.assert_array_equal(counts, np.bincount(values % 16, minlength=16).astype(np.uint32))


def test_warp_sum_dot(zoo):
    rng = np.random.default_rng(6)
    rows, k = 64, 200
    a = rng.standard_normal((rows, k), dtype=np.float32)
    b = rng.standard_normal((rows, k), dtype=np.float32)
    out = np.zeros(rows, np.float32)
    zoo["warp_dot"][(rows, 1, 1), (32, 1, 1)](out, a, b, k)
    np.testing.assert_allclose(out, (a * b).sum(axis=1), atol=1e-3, rtol=1e-4)


def test_device_fn_and_control_flow(zoo):
    rng = np.random.default_rng(7)
    a = (rng.random(4096) * 50.0).astype(np.float32)
    a[::97] *= -1
    out = np.full_like(a, np.nan)
    zoo["cbrt_pos"][(32, 1, 1), (128, 1, 1)](out, a)
    expected = np.where(a <= 0, 0.0, np.cbrt(np.maximum(a, 0))).astype(np.float32)
    np.testing.assert_allclose(out, expected, atol=1e-4, rtol=1e-4)


def test_read_only_kernel_copies_nothing_back(zoo):
    a = np.arange(64, dtype=np.float32)
    b = np.ones(64, np.float32)
    before = (a.copy(), b.copy())
    zoo["read_only"][(1, 1, 1), (64, 1, 1)](a, b)
    np.testing.assert_array_equal(a, before[0])
    np.testing.assert_array_equal(b, before[1])


def test_library_kernels_drop_in():
    rng = np.random.default_rng(8)
    a = rng.standard_normal((512, 512), dtype=np.float32)
    b = rng.standard_normal((512, 512), dtype=np.float32)
    c = np.zeros_like(a)
    tk.kernels.matrix_add((512, 512))(c, a, b)
    np.testing.assert_array_equal(c, a + b)
    a2 = rng.standard_normal((128, 128), dtype=np.float32)
    b2 = rng.standard_normal((128, 128), dtype=np.float32)
    c2 = np.zeros((128, 128), np.float32)
    tk.kernels.matmul(128, 128, 128)(c2, a2, b2)
    np.testing.assert_allclose(c2, a2 @ b2, atol=1e-3, rtol=1e-3)


def test_device_arrays_skip_copies():
    rng = np.random.default_rng(9)
    a = rng.standard_normal(1 << 20, dtype=np.float32)
    b = rng.standard_normal(1 << 20, dtype=np.float32)
    da, db = tk.runtime.to_device(a), tk.runtime.to_device(b)
    dc = tk.runtime.empty(a.shape, np.float32)
    tk.kernels.matrix_add(a.shape)(dc, da, db)
    np.testing.assert_array_equal(dc.to_host(), a + b)
