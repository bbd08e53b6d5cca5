"""The NVLink multicast buffer C-ABI (thork_mc_*) and the multimem fused
GEMM epilogue on one GPU: a multicast object whose only member is this GPU
(skipped where the driver refuses a one-GPU group, as driver 580 does).
A store through the multicast view lands in this GPU's memory, so the
result read through the ordinary view must equal the plain GEMM's bit for
bit (same 128 x 256 tiles).  Multi-GPU groups are covered by
tests/test_gpu_fused_gather.py."""

import ctypes

import numpy as np
import pytest

import thork_b200 as tk
from oracle import oracle

pytestmark = pytest.mark.gpu


def _supported():
    from thork_b200 import dist
    tk.runtime.get_device()
    return dist.multicast_supported()


@pytest.mark.parametrize("dtype", ["bf16", "e4m3"])
def test_multimem_epilogue_on_a_one_gpu_group(dtype):
    if not _supported():
        pytest.skip("NVLink multicast not supported here")
    rt = tk.runtime
    L = rt.lib()
    m, n, k = 512, 768, 512
    a, b = oracle.gemm_inputs(m, n, k, seed=41)
    if dtype == "bf16":
        qa, qb = oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(b)
        sa = sb = 1.0
    else:
        qa, sa = oracle.quantize_e4m3(a)
        qb, sb = oracle.quantize_e4m3(b)
    A, B = rt.to_device(qa), rt.to_device(qb)
    want = rt.empty((m, n), np.uint16)
    if dtype == "bf16":
        rt.check(L.thork_gemm_bf16(A.ptr, B.ptr, want.ptr, m, n, k, 1, None))
    else:
        rt.check(L.thork_gemm_e4m3(A.ptr, B.ptr, want.ptr, m, n, k, sa, sb, 1, None))
    obj, fd, size = ctypes.c_void_p(), ctypes.c_int(), ctypes.c_size_t()
    rc = L.thork_mc_create(m * n * 2, 1, ctypes.byref(obj), ctypes.byref(fd), ctypes.byref(size))
    if rc != 0 and "CUDA_ERROR_INVALID_VALUE" in rt.last_error():
        pytest.skip("this driver refuses a multicast group of one GPU")
    rt.check(rc)
    try:
        assert size.value >= m * n * 2 and fd.value >= 0
        rt.check(L.thork_mc_add_device(obj))
        local, multi = ctypes.c_void_p(), ctypes.c_void_p()
        rt.check(L.thork_mc_bind(obj, ctypes.byref(local), ctypes.byref(multi)))
        rt.check(L.thork_memset(local, 0x7E, size.value, None))
        rt.synchronize()
        # two row blocks, as two ranks of a group would write them
        for row0, rows in ((0, 320), (320, m - 320)):
            a_rows = rt.to_device(np.ascontiguousarray(qa[row0:row0 + rows]))
            if dtype == "bf16":
                rc = L.thork_gemm_bf16_allgather_mc(a_rows.ptr, B.ptr, multi, rows, n, k, row0, None)
            else:
                rc = L.thork_gemm_e4m3_allgather_mc(a_rows.ptr, B.ptr, multi, rows, n, k, row0, sa, sb,
                                                    None)
            rt.check(rc)
            rt.synchronize()
        got = np.empty((m, n), np.uint16)
        rt.copy_dtoh(got, local.value)
        np.testing.assert_array_equal(got, want.to_host())
        assert rt.kernel_status() == 0
    finally:
        rt.check(L.thork_mc_release(obj))
