"""Oracle pins (CPU): the oracle against the reference's own helpers and the
third-party format it follows, via the committed golden fixtures."""

import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_bf16_rounding_matches_reference_helper():
    g = np.load(os.path.join(GOLDEN, "bf16_rne.npz"))
    x = g["x_bits"].view(np.float32)
    bits = oracle.f32_to_bf16_bits(x)
    np.testing.assert_array_equal(bits, g["bf16_bits"])
    np.testing.assert_array_equal(oracle.bf16_bits_to_f32(bits).view(np.uint32), g["widened_bits"])


def test_bf16_rounding_matches_ml_dtypes_on_finite_values():
    ml = pytest.importorskip("ml_dtypes")
    g = np.load(os.path.join(GOLDEN, "bf16_rne.npz"))
    x = g["x_bits"].view(np.float32)
    x = x[np.isfinite(x)]
    ours = oracle.f32_to_bf16_bits(x)
    theirs = x.astype(ml.bfloat16).view(np.uint16)
    # the two agree except where rounding overflows to infinity (identical
    # bits there too) — i.e. everywhere on finite inputs
    np.testing.assert_array_equal(ours, theirs)


def test_e4m3_quantiser_matches_ml_dtypes_sweep():
    g = np.load(os.path.join(GOLDEN, "e4m3_sweep.npz"))
    x = g["x"]
    ours = oracle.f32_to_e4m3_bits(x)
    ref = g["e4m3_bits"]
    # ml_dtypes maps |x| in (464, ...) to NaN; the sweep stops at 464, where
    # both round to the largest finite value or to +-448
    np.testing.assert_array_equal(ours, ref)
    assert float(g["max_finite"]) == oracle.E4M3_MAX


def test_e4m3_table_roundtrip():
    codes = np.arange(256, dtype=np.uint8)
    vals = oracle.e4m3_bits_to_f32(codes)
    finite = np.isfinite(vals)
    back = oracle.f32_to_e4m3_bits(vals[finite])
    # every finite code maps back to itself (zero keeps its sign)
    np.testing.assert_array_equal(back, codes[finite])


def test_e4m3_saturates_above_max():
    big = np.array([448.0, 460.0, 464.0, 500.0, 1e6, -1e6], np.float32)
    vals = oracle.e4m3_bits_to_f32(oracle.f32_to_e4m3_bits(big))
    np.testing.assert_array_equal(np.abs(vals), np.full(6, 448.0, np.float32))


def test_quantize_scale_is_amax_over_448():
    x = np.random.default_rng(0).standard_normal((64, 64)).astype(np.float32)
    q, s = oracle.quantize_e4m3(x)
    assert s == np.float32(np.abs(x).max() / 448.0)
    deq = oracle.e4m3_bits_to_f32(q) * s
    assert np.max(np.abs(deq - x)) <= np.abs(x).max() * 2.0 ** -4 + 1e-6


def test_max_rel_err_definition():
    r = np.array([[1.0, -4.0], [2.0, 0.0]], np.float32)
    c = r + np.array([[0.0, 0.02], [0.0, -0.04]], np.float32)
    assert abs(oracle.max_rel_err(c, r) - 0.01) < 1e-7


def test_seeded_inputs_are_deterministic():
    a1, b1 = oracle.gemm_inputs(8, 16, 32, seed=0)
    a2, b2 = oracle.gemm_inputs(8, 16, 32, seed=0)
    np.testing.assert_array_equal(a1, a2)
    np.testing.assert_array_equal(b1, b2)
    x, w = oracle.skinny_inputs(2, n=64, k=32)
    assert w.shape == (32, 64) and x.shape == (2, 32)
    assert abs(float(w.std()) - 0.02) < 0.005


def test_product_rounding_helpers_match_the_oracle():
    """The package's own host-side converters (used to prepare bf16 / e4m3
    inputs) give the same bytes as the oracle's restatement of the
    reference's rounding, including ties, subnormals and saturation."""
    from thork_b200 import dtypes
    rng = np.random.default_rng(5)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32),
        (rng.standard_normal(2000) * 1e-39).astype(np.float32),   # subnormals
        np.array([0.0, -0.0, 1.0, -1.0, 3.0e38, -3.0e38, 1e-45], np.float32),
        np.frombuffer(rng.integers(0, 2**32, 4000, dtype=np.uint32).astype(np.uint32).tobytes(),
                      np.float32),
    ])
    x = x[np.isfinite(x)]
    np.testing.assert_array_equal(dtypes.to_bf16_bits(x), oracle.f32_to_bf16_bits(x))
    np.testing.assert_array_equal(dtypes.from_bf16_bits(oracle.f32_to_bf16_bits(x)),
                                  oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(x)))
    y = rng.standard_normal((64, 96)).astype(np.float32) * 7.0
    qp, sp = dtypes.quantize_e4m3(y)
    qo, so = oracle.quantize_e4m3(y)
    assert np.float32(sp) == np.float32(so)
    np.testing.assert_array_equal(np.asarray(qp).view(np.uint8), np.asarray(qo).view(np.uint8))
