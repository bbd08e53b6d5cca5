"""GPU parity: tcgen05 GEMMs against the oracle (NumPy fp32 matmul of the
identically rounded inputs, reference ``tests/test_kittens.py:20-36, 101``).

Tolerance (the target specification): max|C - R| / max|R| <= 1e-2 for bf16 and
FP8 e4m3.  Observed errors are ~1e-3 (bf16 output rounding).
"""

import numpy as np
import pytest

import thork_b200 as tk
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _bf16_case(m, n, k, seed=0):
    a, b = oracle.gemm_inputs(m, n, k, seed=seed)
    return oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(b)


def _run_bf16(m, n, k, variant="auto", seed=0):
    a16, b16 = _bf16_case(m, n, k, seed)
    c16 = np.zeros((m, n), np.uint16)
    tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant=variant)(c16, a16, b16)
    ref = oracle.gemm_bf16_ref(a16, b16)
    return oracle.bf16_bits_to_f32(c16), ref


SHAPES = [(128, 256, 64), (256, 256, 256), (200, 264, 136), (1024, 512, 320), (384, 1280, 1024),
          (129, 8, 8), (640, 384, 4096)]


@pytest.mark.parametrize("variant", ["gemm", "gemm2"])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_bf16_shapes(m, n, k, variant):
    c, ref = _run_bf16(m, n, k, variant=variant)
    err = oracle.max_rel_err(c, ref)
    assert err <= TOL, f"max rel err {err:.3e}"
    assert np.isfinite(c).all()


@pytest.mark.parametrize("variant", ["gemm", "gemm2"])
def test_gemm_bf16_config1_4096(variant):
    c, ref = _run_bf16(4096, 4096, 4096, variant=variant)
    err = oracle.max_rel_err(c, ref)
    assert err <= TOL, f"max rel err {err:.3e}"
    # the reference tests' own elementwise check, for information: every
    # element within bf16 output rounding of the fp32 result
    np.testing.assert_allclose(c, ref, atol=2e-1 * float(np.abs(ref).max()) / 64, rtol=2e-2)


@pytest.mark.parametrize("variant", ["gemm", "gemm2"])
def test_gemm_bf16_repeatable_and_linear(variant):
    # determinism: same inputs, same bits; linearity: C(2A) == 2 C(A) exactly
    m = n = k = 512
    a16, b16 = _bf16_case(m, n, k, seed=4)
    mm = tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant=variant)
    c1 = np.zeros((m, n), np.uint16)
    c2 = np.zeros((m, n), np.uint16)
    mm(c1, a16, b16)
    mm(c2, a16, b16)
    np.testing.assert_array_equal(c1, c2)
    a2 = oracle.f32_to_bf16_bits(oracle.bf16_bits_to_f32(a16) * 2)
    c3 = np.zeros((m, n), np.uint16)
    mm(c3, a2, b16)
    np.testing.assert_array_equal(oracle.bf16_bits_to_f32(c3), 2 * oracle.bf16_bits_to_f32(c1))


@pytest.mark.parametrize("variant", ["gemm", "gemm2"])
def test_gemm_bf16_identity_exact(variant):
    # A @ I == A exactly (one nonzero product per output, exact in fp32)
    m, k = 300, 256
    a16, _ = _bf16_case(m, k, k, seed=9)
    eye = oracle.f32_to_bf16_bits(np.eye(k, dtype=np.float32))
    c = np.zeros((m, k), np.uint16)
    tk.kernels.matmul(m, k, k, tk.dt.bfloat16, variant=variant)(c, a16, eye)
    np.testing.assert_array_equal(c, a16)


@pytest.mark.parametrize("variant", ["gemm", "gemm2"])
@pytest.mark.parametrize("m,n,k", [(512, 768, 1024), (300, 272, 160), (128, 256, 128)])
def test_gemm_e4m3(m, n, k, variant):
    a, b = oracle.gemm_inputs(m, n, k, seed=1)
    qa, sa = oracle.quantize_e4m3(a)
    qb, sb = oracle.quantize_e4m3(b)
    c16 = np.zeros((m, n), np.uint16)
    tk.kernels.matmul(m, n, k, tk.dt.float8_e4m3, variant=variant)(c16, qa, qb, sa, sb)
    ref = oracle.gemm_e4m3_ref(qa, sa, qb, sb)
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(c16), ref)
    assert err <= TOL, f"max rel err {err:.3e}"


def test_gemm_e4m3_config3_8192():
    m = n = k = 8192
    a, b = oracle.gemm_inputs(m, n, k, seed=0)
    qa, sa = oracle.quantize_e4m3(a)
    qb, sb = oracle.quantize_e4m3(b)
    c16 = np.zeros((m, n), np.uint16)
    tk.kernels.matmul(m, n, k, tk.dt.float8_e4m3)(c16, qa, qb, sa, sb)
    rows = np.random.default_rng(0).choice(m, 64, replace=False)
    ref = oracle.gemm_e4m3_ref(qa[rows], sa, qb, sb)
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(c16[rows]), ref)
    assert err <= TOL, f"max rel err {err:.3e}"


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 4096), (1000, 784, 1296), (128, 256, 8192),
                                   (300, 4112, 64), (2176, 2560, 512)])
@pytest.mark.parametrize("dtype", ["bf16", "e4m3"])
def test_gemm_stream_k(m, n, k, dtype):
    """Stream-K (equal k-loop shares per SM, split tiles summed in a fixup):
    ragged shapes, a K-only-deep case where every tile is split, a K=64
    case where every CTA holds whole tiles, and the 4096^3 config."""
    a, b = oracle.gemm_inputs(m, n, k, seed=9)
    c16 = np.zeros((m, n), np.uint16)
    if dtype == "bf16":
        a16, b16 = oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(b)
        tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant="gemm_sk")(c16, a16, b16)
        ref = oracle.gemm_bf16_ref(a16, b16)
    else:
        qa, sa = oracle.quantize_e4m3(a)
        qb, sb = oracle.quantize_e4m3(b)
        tk.kernels.matmul(m, n, k, tk.dt.float8_e4m3, variant="gemm_sk")(c16, qa, qb, sa, sb)
        ref = oracle.gemm_e4m3_ref(qa, sa, qb, sb)
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(c16), ref)
    assert err <= TOL, f"max rel err {err:.3e}"
    assert tk.runtime.kernel_status() == 0


def test_gemm_stream_k_is_deterministic_and_linear():
    m, n, k = 1000, 776, 1288
    a16, b16 = _bf16_case(m, n, k, seed=13)
    mm = tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant="gemm_sk")
    c1, c2, c3 = (np.zeros((m, n), np.uint16) for _ in range(3))
    mm(c1, a16, b16)
    mm(c2, a16, b16)
    mm(c3, oracle.f32_to_bf16_bits(oracle.bf16_bits_to_f32(a16) * 2), b16)
    np.testing.assert_array_equal(c1, c2)
    np.testing.assert_array_equal(oracle.bf16_bits_to_f32(c3), 2 * oracle.bf16_bits_to_f32(c1))


@pytest.mark.parametrize("variant", ["auto", "gemm2"])
def test_gemm_bf16_config2_8192(variant):
    """The headline config at full size: a 64-row sample of C against the
    NumPy fp32 product of the bf16-rounded inputs, plus C(2A) == 2 C(A)."""
    m = n = k = 8192
    a16, b16 = _bf16_case(m, n, k, seed=0)
    mm = tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant=variant)
    c16 = np.zeros((m, n), np.uint16)
    mm(c16, a16, b16)
    rows = np.random.default_rng(1).choice(m, 64, replace=False)
    ref = oracle.gemm_bf16_ref(a16[rows], b16)
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(c16[rows]), ref)
    assert err <= TOL, f"max rel err {err:.3e}"
    a2 = oracle.f32_to_bf16_bits(oracle.bf16_bits_to_f32(a16) * 2)
    c2 = np.zeros((m, n), np.uint16)
    mm(c2, a2, b16)
    np.testing.assert_array_equal(oracle.bf16_bits_to_f32(c2), 2 * oracle.bf16_bits_to_f32(c16))


@pytest.mark.parametrize("m", [1, 16, 32, 128])
def test_skinny_gemm_full_size_linear(m):
    """Decode shapes at full size: Y(2X) == 2 Y(X) bit for bit (powers of two
    commute with bf16 rounding and fp32 sums), and repeated calls agree."""
    n, k = 14336, 4096
    x, w = oracle.skinny_inputs(m, n, k, seed=7)
    x16, w16 = oracle.f32_to_bf16_bits(x), oracle.f32_to_bf16_bits(w)
    mm = tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant="skinny")
    y1, y2, y3 = (np.zeros((m, n), np.uint16) for _ in range(3))
    mm(y1, x16, w16)
    mm(y2, x16, w16)
    mm(y3, oracle.f32_to_bf16_bits(oracle.bf16_bits_to_f32(x16) * 2), w16)
    np.testing.assert_array_equal(y1, y2)
    np.testing.assert_array_equal(oracle.bf16_bits_to_f32(y3), 2 * oracle.bf16_bits_to_f32(y1))


@pytest.mark.parametrize("m", [1, 16, 128, 5, 33, 200])
def test_skinny_gemm_bf16(m):
    n, k = (14336, 4096) if m in (1, 16, 128) else (2048, 1024)
    x, w = oracle.skinny_inputs(m, n, k, seed=0)
    x16, w16 = oracle.f32_to_bf16_bits(x), oracle.f32_to_bf16_bits(w)
    y16 = np.zeros((m, n), np.uint16)
    tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant="skinny")(y16, x16, w16)
    ref = oracle.gemm_bf16_ref(x16, w16)
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(y16), ref)
    assert err <= TOL, f"max rel err {err:.3e}"


def test_gemm_bad_shapes_raise():
    with pytest.raises(ValueError):
        tk.kernels.matmul(64, 100, 64, tk.dt.bfloat16)
    with pytest.raises(ValueError):
        tk.kernels.matmul(64, 64, 20, tk.dt.float8_e4m3)


@pytest.mark.parametrize("dtype", ["bf16", "e4m3"])
def test_pipelined_host_path_ragged_chunks(dtype):
    # M = 3000 host arrays: row chunks of 512 (last 440) stream through
    # copy-in / GEMM / copy-out on three streams
    m, n, k = 3000, 512, 384
    a, b = oracle.gemm_inputs(m, n, k, seed=11)
    c16 = np.zeros((m, n), np.uint16)
    if dtype == "bf16":
        a16, b16 = oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(b)
        tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant="gemm")(c16, a16, b16)
        ref = oracle.gemm_bf16_ref(a16, b16)
    else:
        qa, sa = oracle.quantize_e4m3(a)
        qb, sb = oracle.quantize_e4m3(b)
        tk.kernels.matmul(m, n, k, tk.dt.float8_e4m3)(c16, qa, qb, sa, sb)
        ref = oracle.gemm_e4m3_ref(qa, sa, qb, sb)
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(c16), ref)
    assert err <= TOL, f"max rel err {err:.3e}"


@pytest.mark.parametrize("m,n,k", [(20, 14336, 4096), (32, 1024, 512), (1, 4480, 512), (3, 128, 64),
                                   (16, 2048, 8192), (48, 1792, 4096), (64, 3584, 1024),
                                   (40, 1000, 640), (128, 7168, 4096), (100, 3584, 1024),
                                   (65, 4096, 640), (128, 3080, 1000)])
def test_skinny_stream_k_shapes(m, n, k):
    """Decode shapes on both sides of the dispatch rule: stream-K for
    M <= 64 when the 128-column tiles fill at most half of the SMs (most of
    these), one CTA per tile otherwise (M=20 at N=14336, and M > 64)."""
    x, w = oracle.skinny_inputs(m, n, k, seed=5)
    x16, w16 = oracle.f32_to_bf16_bits(x), oracle.f32_to_bf16_bits(w)
    y16 = np.zeros((m, n), np.uint16)
    tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant="skinny")(y16, x16, w16)
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(y16), oracle.gemm_bf16_ref(x16, w16))
    assert err <= TOL, f"max rel err {err:.3e}"


@pytest.mark.parametrize("m,n,k", [(64, 14336, 1024), (65, 2048, 1024), (100, 1160, 768),
                                   (128, 136, 512), (129, 4096, 640), (256, 2304, 512),
                                   (250, 520, 1000)])
def test_skinny_tile_shapes(m, n, k):
    """Decode shapes served one CTA per 128-column tile (M 33..256 with many
    tiles): ragged M leaves part of the X box out of range, ragged N part of
    the last tile's W columns, and K = 1000 ends in a partial 64-wide K
    block.  The output starts as NaN bits so an unwritten element fails."""
    x, w = oracle.skinny_inputs(m, n, k, seed=9)
    x16, w16 = oracle.f32_to_bf16_bits(x), oracle.f32_to_bf16_bits(w)
    y16 = np.full((m, n), 0x7FC0, np.uint16)
    tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant="skinny")(y16, x16, w16)
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(y16), oracle.gemm_bf16_ref(x16, w16))
    assert err <= TOL, f"max rel err {err:.3e}"
    assert tk.runtime.kernel_status() == 0


def test_skinny_stream_k_repeated_calls_are_identical():
    # the split tiles' arrival counters return to zero after every launch, so
    # back-to-back calls (including a different shape in between) agree;
    # N=7168 (56 tiles, under half of the SMs) runs the stream-K kernel
    m, n, k = 16, 7168, 4096
    x, w = oracle.skinny_inputs(m, n, k, seed=6)
    x16, w16 = oracle.f32_to_bf16_bits(x), oracle.f32_to_bf16_bits(w)
    rt = tk.runtime
    dx, dw = rt.to_device(x16), rt.to_device(w16)
    dy = rt.empty((m, n), np.uint16)
    mm = tk.kernels.matmul(m, n, k, tk.dt.bfloat16, variant="skinny")
    outs = []
    for i in range(3):
        mm(dy, dx, dw)
        outs.append(dy.to_host())
        if i == 0:
            other = np.zeros((8, 1024), np.uint16)
            tk.kernels.matmul(8, 1024, 512, tk.dt.bfloat16, variant="skinny")(
                other, x16[:8, :512].copy(), w16[:512, :1024].copy())
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(outs[0]), oracle.gemm_bf16_ref(x16, w16))
    assert err <= TOL


@pytest.mark.parametrize("m", [16, 128])
def test_skinny_static_weights_keep_the_activation_dependency(m):
    """Two decode GEMMs chained on one stream, the second reading the first's
    output as its X, with THORK_SKINNY_W_STATIC on both: W is fetched early,
    X still waits for the previous kernel.  Bit-equal to the chain without
    the flag, and within tolerance of the oracle on the same inputs."""
    rt = tk.runtime
    L = rt.lib()
    k1, n1, n2 = 512, 1024, 2048
    x, w1 = oracle.skinny_inputs(m, n1, k1, seed=11)
    _, w2 = oracle.skinny_inputs(m, n2, n1, seed=12)
    x16, w1_16, w2_16 = (oracle.f32_to_bf16_bits(v) for v in (x, w1, w2))
    X, W1, W2 = rt.to_device(x16), rt.to_device(w1_16), rt.to_device(w2_16)
    s = rt.Stream()
    outs = {}
    for flags in (0, 1):
        Y1, Y2 = rt.empty((m, n1), np.uint16), rt.empty((m, n2), np.uint16)
        for _ in range(3):  # back to back, so the dependent launches overlap
            rt.check(L.thork_skinny_gemm_bf16_ex(X.ptr, W1.ptr, Y1.ptr, m, n1, k1, flags, s.handle))
            rt.check(L.thork_skinny_gemm_bf16_ex(Y1.ptr, W2.ptr, Y2.ptr, m, n2, n1, flags, s.handle))
        s.synchronize()
        outs[flags] = (Y1.to_host(), Y2.to_host())
    assert rt.kernel_status() == 0
    np.testing.assert_array_equal(outs[1][0], outs[0][0])
    np.testing.assert_array_equal(outs[1][1], outs[0][1])
    ref = oracle.gemm_bf16_ref(outs[0][0], w2_16)
    assert oracle.max_rel_err(oracle.bf16_bits_to_f32(outs[1][1]), ref) <= TOL
