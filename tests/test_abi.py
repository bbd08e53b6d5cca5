"""The C-ABI library (CPU): it loads without a GPU, exports every function
include/*.h declares, and the host-side checks behave."""

import ctypes
import os
import re

import pytest

from thork_b200 import runtime as rt

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = []
    for fn in os.listdir(os.path.join(REPO, "include")):
        if fn.endswith(".h"):
            with open(os.path.join(REPO, "include", fn)) as f:
                names += re.findall(r"THORK_API\s+int\s+(thork_\w+)\s*\(", f.read())
    return names


def test_library_loads_and_exports_every_declared_symbol():
    lib = ctypes.CDLL(rt.LIB_PATH)
    names = _declared()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol():
    assert set(_declared()) <= set(rt._SIGNATURES)


def test_version_and_error_text():
    assert rt.lib().thork_version() == 100
    # an invalid argument sets the thread-local error message
    rc = rt.lib().thork_tensor_map_2d(None, 0, None, 1, 1, 16, 1, 1, 0)
    assert rc == rt.ERR_INVALID
    assert "64-byte aligned" in rt.last_error()


def test_nvrtc_is_available():
    a, b = ctypes.c_int(), ctypes.c_int()
    assert rt.lib().thork_nvrtc_version(ctypes.byref(a), ctypes.byref(b)) == 0
    assert (a.value, b.value) >= (12, 8)


def test_library_kernels_reject_bad_shapes_before_touching_a_device():
    L = rt.lib()
    assert L.thork_gemm_bf16(None, None, None, 64, 64, 64, 0, None) == rt.ERR_INVALID
    assert L.thork_gemm_bf16(16, 16, 16, 64, 60, 64, 0, None) == rt.ERR_INVALID
    assert "multiples of 8" in rt.last_error()
    assert L.thork_gemm_e4m3(16, 16, 16, 64, 64, 40, 1.0, 1.0, 0, None) == rt.ERR_INVALID
    assert L.thork_skinny_gemm_bf16(16, 16, 16, 300, 64, 64, None) == rt.ERR_INVALID
    assert L.thork_matrix_add_f32(None, None, None, 0, None) == 0  # empty is a no-op


def test_fused_allgather_and_barrier_reject_bad_arguments_on_the_host():
    L = rt.lib()
    peers = (ctypes.c_void_p * 7)(*([32] * 7))

    def ag(n_peers, row0=0, variant=0, p=peers, flags=None):
        return L.thork_gemm_bf16_allgather(16, 16, 16, p, n_peers, 64, 64, 64, row0, flags, 1,
                                           variant, None)
    assert ag(8) == rt.ERR_INVALID
    assert "n_peers" in rt.last_error()
    assert ag(1, variant=3) == rt.ERR_INVALID
    assert "variant" in rt.last_error()
    assert ag(1, p=(ctypes.c_void_p * 7)(*([40] * 7))) == rt.ERR_INVALID  # not 16-byte aligned
    assert ag(1, row0=-1) == rt.ERR_INVALID
    assert ag(3, variant=2) == rt.ERR_INVALID  # push variant without tile flags
    assert "tile flags" in rt.last_error()
    flags = (ctypes.c_void_p * 8)()
    assert L.thork_peer_barrier(16, flags, 9, 0, 1, None) == rt.ERR_INVALID
    assert L.thork_peer_barrier(16, flags, 2, 2, 1, None) == rt.ERR_INVALID
    assert L.thork_peer_barrier(16, flags, 2, 0, 1, None) == rt.ERR_INVALID  # peer flags NULL
    assert L.thork_ipc_handle(None, None) == rt.ERR_INVALID


def test_nccl_fault_injection_is_host_side(monkeypatch):
    monkeypatch.setenv("THORK_FAULT_NCCL_INIT", "1")
    comm = ctypes.c_void_p()
    uid = (ctypes.c_uint8 * 128)()
    rc = rt.lib().thork_nccl_comm_init_rank(ctypes.byref(comm), 2, uid, 0)
    assert rc == rt.ERR_NCCL
    assert "injected failure" in rt.last_error()


def test_nvrtc_compile_error_is_rewritten_with_python_locations():
    src = "extern \"C\" __global__ void k(float *x)\n{\n    x[0] = undefined_name;\n}\n"
    with pytest.raises(RuntimeError) as ei:
        rt.nvrtc_compile(src, source_map={3: ("user.py", 42)}, use_cache=False)
    msg = str(ei.value)
    assert msg.startswith("NVRTC compile failed")
    assert "generated line 3 -> user.py:42" in msg
