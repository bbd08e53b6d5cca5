"""Copies between pageable NumPy memory and the device through the pinned
staging ring (sizes from just below the 1 MiB threshold to several slots,
odd lengths), on the default stream and on a side stream, bit-exact round
trips; and the drop-in call on pageable arrays above the threshold."""

import numpy as np
import pytest

import thork_b200 as tk
from oracle import oracle

pytestmark = pytest.mark.gpu
rt = tk.runtime


@pytest.mark.parametrize("nbytes", [(1 << 20) - 3, 1 << 20, 3_500_001, 40 * (1 << 20) + 17])
@pytest.mark.parametrize("use_stream", [False, True])
def test_pageable_round_trip_is_exact(nbytes, use_stream):
    rng = np.random.default_rng(nbytes)
    src = rng.integers(0, 256, nbytes, dtype=np.uint8)
    dst = np.zeros_like(src)
    d = rt.empty((nbytes,), np.uint8)
    s = rt.Stream() if use_stream else None
    rt.copy_htod(d.ptr, src, s, sync=False)
    src_copy = src.copy()
    src[:] = 0  # the source may be reused once the copy call returns
    rt.copy_dtoh(dst, d.ptr, s, sync=False)
    if s is not None:
        s.synchronize()
    np.testing.assert_array_equal(dst, src_copy)


def test_back_to_back_staged_copies_keep_order():
    s = rt.Stream()
    bufs = [rt.empty((12 << 20,), np.uint8) for _ in range(3)]
    hs = [np.full(12 << 20, i + 1, np.uint8) for i in range(3)]
    for h, d in zip(hs, bufs):
        rt.copy_htod(d.ptr, h, s, sync=False)
    outs = [np.zeros(12 << 20, np.uint8) for _ in range(3)]
    for o, d in zip(outs, bufs):
        rt.copy_dtoh(o, d.ptr, s, sync=False)
    for i, o in enumerate(outs):
        assert (o == i + 1).all()


def test_dropin_add_on_large_pageable_arrays():
    a, b = oracle.add_inputs((3000, 1001), seed=4)  # 12 MB each, odd sizes
    out = np.zeros_like(a)
    tk.kernels.matrix_add(a.shape)(out, a, b)
    np.testing.assert_array_equal(out, oracle.add_ref(a, b))
