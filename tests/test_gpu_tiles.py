"""GPU parity of the tile-op front end (tk.kittens) lowered to the sm_100a
tile library: register-tile mma.sync, TMA-fed and tcgen05/TMEM matmuls
against the oracle (NumPy fp32 matmul of the bf16-rounded inputs).

Tolerances: the reference tile tests' own check (atol=2e-1, rtol=2e-2 on
0.1*N(0,1) inputs against the unrounded product, ``tests/test_kittens.py:101,
184``) and the north_star bound max|C-R|/max|R| <= 1e-2 against the rounded
inputs."""

import numpy as np
import pytest

import thork_b200 as tk
from oracle import oracle

import tile_kernels

pytestmark = pytest.mark.gpu


def _inputs(m, n, k, seed):
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal((m, k)) * 0.1).astype(np.float32)
    b = (rng.standard_normal((k, n)) * 0.1).astype(np.float32)
    return a, b, oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(b)


def _check(c16, a, b, a16, b16):
    c = oracle.bf16_bits_to_f32(c16)
    np.testing.assert_allclose(c, a @ b, atol=2e-1, rtol=2e-2)
    err = oracle.max_rel_err(c, oracle.gemm_bf16_ref(a16, b16))
    assert err <= 1e-2, f"max rel err {err:.3e}"


@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (64, 96, 256)])
def test_register_tile_matmul(m, n, k):
    a, b, a16, b16 = _inputs(m, n, k, 0)
    c16 = np.zeros((m, n), np.uint16)
    kern = tile_kernels.regtile_matmul(tk)
    kern[(n // 32, m // 32, 1), (32, 1, 1)](a16, b16, c16, k)
    _check(c16, a, b, a16, b16)


@pytest.mark.parametrize("n", [128, 256])
def test_tma_matmul(n):
    a, b, a16, b16 = _inputs(n, n, n, 1)
    c16 = np.zeros((n, n), np.uint16)
    kern = tile_kernels.tma_matmul(tk)
    kern[(n // 64, n // 64, 1), (32, 1, 1)](a16, b16, c16, n)
    _check(c16, a, b, a16, b16)


@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (256, 384, 512)])
def test_tcgen05_matmul(m, n, k):
    a, b, a16, b16 = _inputs(m, n, k, 2)
    d16 = np.zeros((m, n), np.uint16)
    kern = tile_kernels.tcgen05_matmul(tk)
    kern[((m // 128) * (n // 128), 1, 1), (128, 1, 1)](a16, b16, d16, k, n)
    _check(d16, a, b, a16, b16)
    assert tk.runtime.kernel_status() == 0


def test_tile_kernel_uses_ml_dtypes_bf16_arrays():
    ml = pytest.importorskip("ml_dtypes")
    a, b, a16, b16 = _inputs(128, 128, 128, 3)
    c = np.zeros((128, 128), ml.bfloat16)
    kern = tile_kernels.regtile_matmul(tk)
    kern[(4, 4, 1), (32, 1, 1)](a16.view(ml.bfloat16), b16.view(ml.bfloat16), c, 128)
    _check(c.view(np.uint16), a, b, a16, b16)
