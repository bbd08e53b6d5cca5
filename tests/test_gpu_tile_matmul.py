"""GPU parity of tk.kernels.tile_matmul: the warp-specialised tcgen05 tile
matmul written with tk.kittens, in its 1-CTA (128 x 256 tiles) and
cluster-pair (tcgen05 cta_group::2, 256 x 256 tiles) forms.

Tolerance: max|C-R|/max|R| <= 1e-2 against NumPy fp32 matmul of the
bf16-rounded inputs (north_star), plus the reference tile tests' own
``assert_allclose(atol=2e-1, rtol=2e-2)`` on 0.1*N(0,1) inputs
(``tests/test_kittens.py:101``)."""

import numpy as np
import pytest

import thork_b200 as tk
from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _inputs(m, n, k, seed, scale=0.1):
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal((m, k)) * scale).astype(np.float32)
    b = (rng.standard_normal((k, n)) * scale).astype(np.float32)
    return a, b, oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(b)


@pytest.mark.parametrize("ncta", [1, 2])
@pytest.mark.parametrize("m,n,k", [(256, 512, 512), (512, 256, 192), (256, 256, 64),
                                   (768, 1024, 1088)])
def test_tile_matmul_matches_oracle(ncta, m, n, k):
    # K = 64 and 192: fewer k-blocks than stages; K = 1088: a partial last round
    a, b, a16, b16 = _inputs(m, n, k, seed=m + n + k)
    c16 = np.zeros((m, n), np.uint16)
    tk.kernels.tile_matmul(m, n, k, ncta=ncta)(c16, a16, b16)
    c = oracle.bf16_bits_to_f32(c16)
    err = oracle.max_rel_err(c, oracle.gemm_bf16_ref(a16, b16))
    assert err <= TOL, f"ncta={ncta}: max rel err {err:.3e}"
    np.testing.assert_allclose(c, a @ b, atol=2e-1, rtol=2e-2)
    assert tk.runtime.kernel_status() == 0


@pytest.mark.parametrize("ncta", [1, 2])
def test_tile_matmul_4096_device_resident(ncta):
    """The benchmarked size on device arrays: 64 sampled rows against the
    oracle, and C(2A) == 2 C(A) bit for bit over the whole matrix."""
    m = n = k = 4096
    rt = tk.runtime
    a, b, a16, b16 = _inputs(m, n, k, seed=4, scale=1.0)
    A, B = rt.to_device(a16), rt.to_device(b16)
    C = rt.empty((m, n), np.uint16)
    C.zero()
    mm = tk.kernels.tile_matmul(m, n, k, ncta=ncta)
    mm(C, A, B)
    c = C.to_host()
    rows = np.sort(np.random.default_rng(5).choice(m, 64, replace=False))
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(c[rows]), oracle.gemm_bf16_ref(a16[rows], b16))
    assert err <= TOL, f"max rel err {err:.3e}"
    A2 = rt.to_device(oracle.f32_to_bf16_bits(oracle.bf16_bits_to_f32(a16) * 2))
    C2 = rt.empty((m, n), np.uint16)
    mm(C2, A2, B)
    np.testing.assert_array_equal(oracle.bf16_bits_to_f32(C2.to_host()),
                                  2 * oracle.bf16_bits_to_f32(c))
    assert rt.kernel_status() == 0


def test_pair_and_single_cta_agree_bit_for_bit():
    """Both forms accumulate every k-block in the same order in fp32, so
    their bf16 outputs are identical."""
    m, n, k = 512, 512, 1024
    _, _, a16, b16 = _inputs(m, n, k, seed=8, scale=1.0)
    c1, c2 = np.zeros((m, n), np.uint16), np.zeros((m, n), np.uint16)
    tk.kernels.tile_matmul(m, n, k, ncta=1)(c1, a16, b16)
    tk.kernels.tile_matmul(m, n, k, ncta=2)(c2, a16, b16)
    np.testing.assert_array_equal(c1, c2)


def test_prepared_launches_match_dropin_call():
    """Arguments packed once, launches queued asynchronously on a stream,
    give the same bits as the synchronous drop-in call; host arrays are
    refused (a prepared launch copies nothing)."""
    rt = tk.runtime
    m, n, k = 256, 512, 512
    _, _, a16, b16 = _inputs(m, n, k, seed=9, scale=1.0)
    mm = tk.kernels.tile_matmul(m, n, k, ncta=2)
    want = np.zeros((m, n), np.uint16)
    mm(want, a16, b16)
    A, B, C = rt.to_device(a16), rt.to_device(b16), rt.empty((m, n), np.uint16)
    C.zero()
    s = rt.Stream()
    prepared = mm.prepare(C, A, B)
    for _ in range(3):
        prepared.launch(s)
    s.synchronize()
    np.testing.assert_array_equal(C.to_host(), want)
    assert rt.kernel_status() == 0
    with pytest.raises(TypeError, match="DeviceArray"):
        mm.prepare(want, A, B)


@pytest.mark.parametrize("m,n,k", [(2048, 4096, 256), (512, 512, 512), (4096, 4096, 4096)])
def test_persistent_tile_matmul(m, n, k):
    """The persistent form (one CTA per SM, two TMEM accumulators): several
    tiles per CTA at 2048 x 4096 and 4096^3, bit-equal to the one-tile-per-CTA
    form (same 128 x 256 tiles, same k order)."""
    rt = tk.runtime
    _, _, a16, b16 = _inputs(m, n, k, seed=m + k, scale=1.0)
    A, B = rt.to_device(a16), rt.to_device(b16)
    C1, C2 = rt.empty((m, n), np.uint16), rt.empty((m, n), np.uint16)
    tk.kernels.tile_matmul(m, n, k, persistent=True)(C1, A, B)
    tk.kernels.tile_matmul(m, n, k)(C2, A, B)
    c1 = C1.to_host()
    np.testing.assert_array_equal(c1, C2.to_host())
    rows = np.sort(np.random.default_rng(6).choice(m, 64, replace=False))
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(c1[rows]), oracle.gemm_bf16_ref(a16[rows], b16))
    assert err <= TOL, f"max rel err {err:.3e}"
    assert rt.kernel_status() == 0
