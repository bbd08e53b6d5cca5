"""The allocation-free decode GEMM entry point (thork_skinny_gemm_bf16_noalloc).

It serves callers that must not allocate device memory themselves or
through this library (a process whose memory pool owns the GPU, or a path
that cannot take cudaMalloc's device-wide synchronisation).  Its scratch is
a fixed array compiled into libthork_rt.so, shared by every call, and its
bounded-wait status word lives in that array too
(thork_skinny_gemm_bf16_noalloc_status reads it).

The main test makes its no-alloc calls before the allocating entry point
runs in the test, reads the device's free memory around them, then compares
each of two calls in a row with the allocating entry point's output and
with the oracle.  The file is collected last so that a run stopping at the
first failure has run everything else."""

import numpy as np
import pytest

import thork_b200 as tk
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-2


def test_no_alloc_entry_point_matches_allocating_one_twice():
    rt = tk.runtime
    lib = rt.lib()
    rt.get_device()
    m, n, k = 16, 14336, 4096
    x, w = oracle.skinny_inputs(m, n, k, seed=12)
    x16, w16 = oracle.f32_to_bf16_bits(x), oracle.f32_to_bf16_bits(w)
    dx, dw = rt.to_device(x16), rt.to_device(w16)
    ys = [rt.empty((m, n), np.uint16) for _ in range(2)]
    for y in ys:
        y.zero()
    rt.synchronize()
    # a clean slate for the sticky status word (an earlier test may have run it)
    rt.noalloc_status(clear=True)

    # the first call on a device may load the library's module (and with it the
    # static scratch array); the two calls after it are the ones measured
    rt.check(lib.thork_skinny_gemm_bf16_noalloc(dx.ptr, dw.ptr, ys[0].ptr, m, n, k, None))
    rt.synchronize()
    free_before, _ = rt.mem_info()
    for y in ys:
        rt.check(lib.thork_skinny_gemm_bf16_noalloc(dx.ptr, dw.ptr, y.ptr, m, n, k, None))
        rt.synchronize()
        assert rt.noalloc_status(clear=False) == 0, "a bounded wait expired in a no-alloc call"
    free_after, _ = rt.mem_info()
    assert free_after == free_before, \
        f"device free memory changed across no-alloc calls: {free_before} -> {free_after}"

    y_ref = rt.empty((m, n), np.uint16)
    rt.check(lib.thork_skinny_gemm_bf16(dx.ptr, dw.ptr, y_ref.ptr, m, n, k, None))
    rt.synchronize()
    ref = oracle.bf16_bits_to_f32(y_ref.to_host())
    exact = oracle.gemm_bf16_ref(x16, w16)
    for call, y in enumerate(ys):
        got = oracle.bf16_bits_to_f32(y.to_host())
        err = oracle.max_rel_err(got, ref)
        assert err <= TOL, f"call {call}: max rel err vs allocating entry point {err:.3e}"
        assert oracle.max_rel_err(got, exact) <= TOL
    assert rt.noalloc_status(clear=True) == 0
    assert rt.kernel_status() == 0


def test_no_alloc_entry_point_rejects_oversized_requests():
    rt = tk.runtime
    lib = rt.lib()
    rt.get_device()
    dummy = rt.empty((1024,), np.uint16)
    assert lib.thork_skinny_gemm_bf16_noalloc(dummy.ptr, dummy.ptr, dummy.ptr, 33, 1024, 512, None) \
        == rt.ERR_INVALID
    assert "M must be <= 32" in rt.last_error()
    # more than 16384 output tiles of 128 columns: the tile counters exceed the array
    # (rejected on the host before anything is launched)
    assert lib.thork_skinny_gemm_bf16_noalloc(dummy.ptr, dummy.ptr, dummy.ptr, 32, 16385 * 128, 512,
                                              None) == rt.ERR_INVALID
    assert "scratch array" in rt.last_error()
