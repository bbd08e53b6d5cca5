"""GPU parity: elementwise fp32 add, bit-exact against the oracle (NumPy
``A + B``, the reference's check in ``tests/test_thork.py:6-35``)."""

import numpy as np
import pytest

import thork_b200 as tk
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_library_matrix_add_config0_bit_exact():
    a, b = oracle.add_inputs((1024, 1024), seed=0)
    c = np.zeros_like(a)
    tk.kernels.matrix_add((1024, 1024))(c, a, b)
    np.testing.assert_array_equal(c, oracle.add_ref(a, b))


def test_traced_matrix_add_readme_kernel_bit_exact():
    a, b = oracle.add_inputs((1024, 1024), seed=1)
    c = np.zeros_like(a)

    @tk.jit
    def add(out: tk.DevicePointer[tk.dt.float32], x: tk.DevicePointer[tk.dt.float32],
            y: tk.DevicePointer[tk.dt.float32], bid: tk.Uint[tk.BlockIdx],
            tid: tk.Uint[tk.ThreadIdx], bdm: tk.Uint[tk.BlockDim]):
        i = bid * bdm + tid
        out[i] = x[i] + y[i]

    add[(a.size // 128, 1, 1), (128, 1, 1)](c, a, b)
    np.testing.assert_array_equal(c, oracle.add_ref(a, b))


@pytest.mark.parametrize("n", [1, 3, 4, 5, 127, 1000, 4099, 1 << 20, (1 << 22) + 7])
def test_matrix_add_ragged_sizes(n):
    rng = np.random.default_rng(n)
    a = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    c = np.full(n, np.nan, np.float32)
    tk.kernels.matrix_add((n,))(c, a, b)
    np.testing.assert_array_equal(c, oracle.add_ref(a, b))


def test_matrix_add_special_values_bit_exact():
    vals = np.array([0.0, -0.0, 1e-45, -1e-45, 1.17549435e-38, 3.4028235e38, -3.4028235e38,
                     np.inf, -np.inf, 1.0, -1.0, 2.0 ** -149, 0.1, 1e30], np.float32)
    a = np.repeat(vals, len(vals))
    b = np.tile(vals, len(vals))
    c = np.zeros_like(a)
    tk.kernels.matrix_add((a.size,))(c, a, b)
    with np.errstate(over="ignore", invalid="ignore"):
        ref = oracle.add_ref(a, b)
    # bit-exact everywhere except NaN payloads (inf + -inf), which IEEE 754
    # leaves unspecified: NumPy yields 0xffc00000, the GPU 0x7fffffff
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(c), nan)
    np.testing.assert_array_equal(c.view(np.uint32)[~nan], ref.view(np.uint32)[~nan])


def test_matrix_add_unaligned_views_use_scalar_path():
    # device buffers are always aligned; a DeviceArray offset exercises the
    # unaligned branch through the C-ABI directly
    rt = tk.runtime
    n = 10001
    rng = np.random.default_rng(7)
    a = rng.standard_normal(n + 1, dtype=np.float32)
    b = rng.standard_normal(n + 1, dtype=np.float32)
    da, db = rt.to_device(a), rt.to_device(b)
    dc = rt.empty((n + 1,), np.float32)
    rt.check(rt.lib().thork_matrix_add_f32(dc.ptr + 4, da.ptr + 4, db.ptr + 4, n, None))
    rt.synchronize()
    out = dc.to_host()
    np.testing.assert_array_equal(out[1:], oracle.add_ref(a[1:], b[1:]))


def test_matrix_add_large_property():
    # 2^26 elements (768 MiB of traffic): commutativity and x + 0 == x
    n = 1 << 26
    rng = np.random.default_rng(3)
    a = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    c1 = np.empty_like(a)
    c2 = np.empty_like(a)
    add = tk.kernels.matrix_add((n,))
    add(c1, a, b)
    add(c2, b, a)
    np.testing.assert_array_equal(c1, c2)
    np.testing.assert_array_equal(c1[::9973], oracle.add_ref(a[::9973], b[::9973]))
    z = np.zeros_like(a)
    add(c2, a, z)
    np.testing.assert_array_equal(c2, a)


def test_matrix_add_float16_traced_path():
    rng = np.random.default_rng(5)
    a = rng.standard_normal(5000).astype(np.float16)
    b = rng.standard_normal(5000).astype(np.float16)
    c = np.zeros_like(a)
    tk.kernels.matrix_add((5000,), tk.dt.float16)(c, a, b)
    np.testing.assert_array_equal(c, (a + b).astype(np.float16))
