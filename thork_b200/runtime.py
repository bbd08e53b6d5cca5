"""Host runtime: a ctypes binding of ``libthork_rt.so`` (include/thork_rt.h).

Replaces the reference's cuda-python runtime (``src/thork/runtime.py``):

* device/context set-up (``runtime.py:85-105``) -> ``get_device``; any
  device, not only device 0 (``set_device``);
* NVRTC compilation (``runtime.py:373-421``) -> ``compile_source``, which
  builds a **cubin for sm_100a** (not PTX for ``compute_<cap>``) and keeps a
  content-addressed disk cache; the nvcc/ThunderKittens route
  (``runtime.py:245-370``) is gone: tile kernels compile through NVRTC too;
* argument validation, per-call copy-in / launch / synchronise / copy-back
  of written buffers / free (``runtime.py:431-700``) -> ``dispatch``, with the
  same checks, error types and messages.  Device buffers come from a small
  caching allocator instead of a cuMemAlloc/cuMemFree pair per argument.

There is no CPU fallback: if the library or a GPU is missing, calls raise.
"""

import ctypes
import hashlib
import os
import re
import struct
import threading
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import dtypes as dt
from . import ir

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libthork_rt.so")
DEVICE_INCLUDE = os.path.join(PKG_DIR, "csrc", "device")
ARCH = "sm_100a"

# status codes (include/thork_rt.h)
THORK_OK = 0
ERR_CUDA, ERR_NVRTC, ERR_NCCL, ERR_INVALID, ERR_KERNEL, ERR_UNAVAILABLE = 1, 2, 3, 4, 5, 6
DT_CODE = {"uint8": 0, "uint16": 1, "uint32": 2, "float32": 3, "bfloat16": 4, "float16": 5,
           "float8_e4m3": 6, "int32": 2}

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_i = ctypes.c_int
_u = ctypes.c_uint
_u64 = ctypes.c_uint64
_u32 = ctypes.c_uint32
_pvp = ctypes.POINTER(ctypes.c_void_p)

# (name, argtypes) of every exported function
_SIGNATURES = {
    "thork_version": [],
    "thork_last_error": [ctypes.c_char_p, _sz],
    "thork_device_count": [ctypes.POINTER(_i)],
    "thork_init": [_i],
    "thork_device_attr": [_i, _i, ctypes.POINTER(_i)],
    "thork_device_synchronize": [],
    "thork_malloc": [_sz, _pvp],
    "thork_free": [_vp],
    "thork_host_alloc": [_sz, _pvp],
    "thork_host_free": [_vp],
    "thork_memcpy_htod": [_vp, _vp, _sz, _vp, _i],
    "thork_memcpy_dtoh": [_vp, _vp, _sz, _vp, _i],
    "thork_memcpy_dtod": [_vp, _vp, _sz, _vp],
    "thork_memset": [_vp, _i, _sz, _vp],
    "thork_mem_info": [ctypes.POINTER(_sz), ctypes.POINTER(_sz)],
    "thork_stream_create": [_pvp],
    "thork_stream_destroy": [_vp],
    "thork_stream_synchronize": [_vp],
    "thork_event_create": [_pvp],
    "thork_event_destroy": [_vp],
    "thork_event_record": [_vp, _vp],
    "thork_event_synchronize": [_vp],
    "thork_event_elapsed_ms": [_vp, _vp, ctypes.POINTER(ctypes.c_float)],
    "thork_stream_wait_event": [_vp, _vp],
    "thork_nvrtc_version": [ctypes.POINTER(_i), ctypes.POINTER(_i)],
    "thork_nvrtc_compile": [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                            ctypes.POINTER(ctypes.c_char_p), _i, _pvp, ctypes.POINTER(_sz),
                            ctypes.POINTER(ctypes.c_void_p)],
    "thork_buffer_free": [_vp],
    "thork_module_load": [_vp, _pvp],
    "thork_module_unload": [_vp],
    "thork_module_get_function": [_vp, ctypes.c_char_p, _pvp],
    "thork_function_set_max_dynamic_smem": [_vp, _i],
    "thork_launch": [_vp, ctypes.POINTER(_u), ctypes.POINTER(_u), ctypes.POINTER(_u), _u, _vp, _pvp],
    "thork_tensor_map_2d": [_vp, _i, _vp, _u64, _u64, _u64, _u32, _u32, _i],
    "thork_kernel_status": [ctypes.POINTER(_u), _i],
    "thork_status_pointer": [_pvp],
    "thork_matrix_add_f32": [_vp, _vp, _vp, _sz, _vp],
    "thork_gemm_bf16": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "thork_gemm_e4m3": [_vp, _vp, _vp, _i, _i, _i, ctypes.c_float, ctypes.c_float, _i, _vp],
    "thork_skinny_gemm_bf16": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "thork_skinny_gemm_bf16_noalloc": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "thork_skinny_gemm_bf16_noalloc_status": [ctypes.POINTER(_u), _i, _vp],
    "thork_skinny_gemm_bf16_ex": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "thork_gemm_bf16_allgather": [_vp, _vp, _vp, _pvp, _i, _i, _i, _i, _i, _vp, ctypes.c_uint, _i,
                                  _vp],
    "thork_gemm_e4m3_allgather": [_vp, _vp, _vp, _pvp, _i, _i, _i, _i, _i, _vp, ctypes.c_uint,
                                  ctypes.c_float, ctypes.c_float, _i, _vp],
    "thork_peer_barrier": [_vp, _pvp, _i, _i, ctypes.c_uint, _vp],
    "thork_ipc_handle": [_vp, _vp],
    "thork_ipc_open": [_vp, _pvp],
    "thork_ipc_close": [_vp],
    "thork_gemm_bf16_allgather_mc": [_vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "thork_gemm_e4m3_allgather_mc": [_vp, _vp, _vp, _i, _i, _i, _i, ctypes.c_float,
                                     ctypes.c_float, _vp],
    "thork_mc_supported": [ctypes.POINTER(_i)],
    "thork_mc_create": [_sz, _i, _pvp, ctypes.POINTER(_i), ctypes.POINTER(_sz)],
    "thork_mc_import": [_i, _sz, _pvp],
    "thork_mc_add_device": [_vp],
    "thork_mc_bind": [_vp, _pvp, _pvp],
    "thork_mc_release": [_vp],
    "thork_nccl_get_unique_id": [_vp],
    "thork_nccl_comm_init_rank": [_pvp, _i, _vp, _i],
    "thork_nccl_comm_destroy": [_vp],
    "thork_nccl_allgather": [_vp, _vp, _sz, _i, _vp, _vp],
    "thork_nccl_allreduce_sum": [_vp, _sz, _i, _vp, _vp],
}

_lib_handle = None
_lib_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load (once) the in-tree ``libthork_rt.so``; raise if it is not built."""
    global _lib_handle
    if _lib_handle is not None:
        return _lib_handle
    with _lib_lock:
        if _lib_handle is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"thork_b200 native library not found at {LIB_PATH}; build it with "
                    "`python -m thork_b200.build` (there is no CPU fallback)")
            h = ctypes.CDLL(LIB_PATH)
            for name, argtypes in _SIGNATURES.items():
                fn = getattr(h, name)
                fn.argtypes = argtypes
                fn.restype = ctypes.c_int
            _lib_handle = h
    return _lib_handle


def last_error() -> str:
    buf = ctypes.create_string_buffer(4096)
    lib().thork_last_error(buf, len(buf))
    return buf.value.decode("utf-8", errors="replace")


class CudaError(RuntimeError):
    """A failed runtime call; ``code`` is the thork status code."""

    def __init__(self, msg: str, code: int):
        super().__init__(msg)
        self.code = code


def check(rc: int, what: str = "") -> None:
    if rc != THORK_OK:
        msg = last_error()
        if what and what not in msg:
            msg = f"{msg} [{what}]"
        raise CudaError(msg, rc)


# --------------------------------------------------------------------------
# device / context
# --------------------------------------------------------------------------
_state = threading.local()
_initialised: Dict[int, bool] = {}
_default_device = int(os.environ.get("THORK_DEVICE", "0"))


def device_count() -> int:
    n = ctypes.c_int(0)
    check(lib().thork_device_count(ctypes.byref(n)), "device_count")
    return n.value


def set_device(dev: int) -> None:
    """Select the device this thread launches on (default ``$THORK_DEVICE`` or 0)."""
    check(lib().thork_init(int(dev)), f"init device {dev}")
    _initialised[int(dev)] = True
    _state.device = int(dev)


def get_device() -> int:
    """Initialise (once per thread) and return the current device index."""
    dev = getattr(_state, "device", None)
    if dev is None:
        set_device(_default_device)
        dev = _state.device
    return dev


def device_attr(attr: int, dev: Optional[int] = None) -> int:
    v = ctypes.c_int(0)
    check(lib().thork_device_attr(get_device() if dev is None else dev, attr, ctypes.byref(v)))
    return v.value


def get_compute_capability() -> str:
    """``"<major><minor>"`` of the current device, e.g. ``"100"`` on B200."""
    return f"{device_attr(0)}{device_attr(1)}"


def sm_count() -> int:
    return device_attr(2)


def max_dynamic_shared_size() -> int:
    """Opt-in dynamic shared memory per block minus a 1 KiB reserve
    (reference ``runtime.py:172-186``)."""
    return device_attr(3) - 1024


def synchronize() -> None:
    get_device()
    check(lib().thork_device_synchronize(), "device synchronize")


def kernel_status(clear: bool = True) -> int:
    """Status word of the current device: non-zero after a bounded wait in a
    kernel expired (code in bits 0-7, wait site in bits 8-15)."""
    get_device()
    v = ctypes.c_uint(0)
    check(lib().thork_kernel_status(ctypes.byref(v), 1 if clear else 0), "kernel status")
    return v.value


def check_kernel_status(what: str) -> None:
    st = kernel_status(clear=True)
    if st:
        raise CudaError(
            f"kernel {what} reported status 0x{st:x} (a bounded wait expired at site "
            f"{(st >> 8) & 0xFF})", ERR_KERNEL)


# --------------------------------------------------------------------------
# streams and events
# --------------------------------------------------------------------------
class Stream:
    def __init__(self):
        get_device()
        h = ctypes.c_void_p()
        check(lib().thork_stream_create(ctypes.byref(h)), "stream create")
        self.handle = h.value

    def synchronize(self) -> None:
        check(lib().thork_stream_synchronize(self.handle), "stream synchronize")

    def wait(self, event: "Event") -> None:
        """Order later work on this stream after ``event``."""
        check(lib().thork_stream_wait_event(self.handle, event.handle), "stream wait event")

    def close(self) -> None:
        if self.handle:
            lib().thork_stream_destroy(self.handle)
            self.handle = None


class Event:
    def __init__(self):
        get_device()
        h = ctypes.c_void_p()
        check(lib().thork_event_create(ctypes.byref(h)), "event create")
        self.handle = h.value

    def record(self, stream: Optional["Stream"] = None) -> None:
        check(lib().thork_event_record(self.handle, stream.handle if stream else None), "event record")

    def synchronize(self) -> None:
        check(lib().thork_event_synchronize(self.handle), "event synchronize")

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float()
        check(lib().thork_event_elapsed_ms(self.handle, end.handle, ctypes.byref(ms)), "elapsed")
        return float(ms.value)

    def close(self) -> None:
        if self.handle:
            lib().thork_event_destroy(self.handle)
            self.handle = None


def _dispatch_stream() -> Stream:
    s = getattr(_state, "stream", None)
    if s is None:
        s = Stream()
        _state.stream = s
    return s


# --------------------------------------------------------------------------
# memory
# --------------------------------------------------------------------------
class _Pool:
    """Size-bucketed cache of device allocations (per device).

    ``cudaFree`` synchronises the device and ``cudaMalloc`` costs tens of
    microseconds, so buffers released by ``dispatch`` are kept for reuse up to
    ``THORK_POOL_BYTES`` (default 8 GiB) per device.
    """

    def __init__(self):
        self._free: Dict[Tuple[int, int], List[int]] = {}
        self._cached = 0
        self._limit = int(os.environ.get("THORK_POOL_BYTES", str(8 << 30)))
        self._lock = threading.Lock()

    @staticmethod
    def _round(n: int) -> int:
        n = max(int(n), 512)
        if n <= (1 << 20):
            return 1 << (n - 1).bit_length()
        return (n + (1 << 20) - 1) & ~((1 << 20) - 1)

    def alloc(self, nbytes: int) -> Tuple[int, int]:
        dev = get_device()
        size = self._round(nbytes)
        with self._lock:
            lst = self._free.get((dev, size))
            if lst:
                self._cached -= size
                return lst.pop(), size
        p = ctypes.c_void_p()
        rc = lib().thork_malloc(size, ctypes.byref(p))
        if rc != THORK_OK:
            self.trim()
            check(lib().thork_malloc(size, ctypes.byref(p)), f"malloc {size} bytes")
        return p.value, size

    def release(self, ptr: int, size: int, dev: int) -> None:
        with self._lock:
            if self._cached + size <= self._limit:
                self._free.setdefault((dev, size), []).append(ptr)
                self._cached += size
                return
        lib().thork_free(ptr)

    def trim(self) -> None:
        with self._lock:
            for lst in self._free.values():
                for ptr in lst:
                    lib().thork_free(ptr)
            self._free.clear()
            self._cached = 0


_pool = _Pool()


class DeviceBuffer:
    """An owned device allocation of at least ``nbytes`` bytes."""

    __slots__ = ("ptr", "nbytes", "_size", "_dev")

    def __init__(self, nbytes: int):
        self.nbytes = int(nbytes)
        self.ptr, self._size = _pool.alloc(self.nbytes)
        self._dev = get_device()

    def free(self) -> None:
        if self.ptr:
            _pool.release(self.ptr, self._size, self._dev)
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class DeviceArray:
    """A device-resident array (shape, dtype) usable as a kernel argument
    without host copies.  ``to_host()`` copies it back into NumPy."""

    def __init__(self, shape, dtype, buffer: Optional[DeviceBuffer] = None):
        self.shape = tuple(int(s) for s in shape)
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        self.buffer = buffer if buffer is not None else DeviceBuffer(self.nbytes)

    @property
    def ptr(self) -> int:
        return self.buffer.ptr

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @classmethod
    def from_host(cls, arr: np.ndarray, stream: Optional[Stream] = None) -> "DeviceArray":
        arr = np.ascontiguousarray(arr)
        d = cls(arr.shape, arr.dtype)
        copy_htod(d.ptr, arr, stream)
        return d

    def to_host(self, out: Optional[np.ndarray] = None, stream: Optional[Stream] = None) -> np.ndarray:
        if out is None:
            out = np.empty(self.shape, self.dtype)
        copy_dtoh(out, self.ptr, stream)
        return out

    def zero(self, stream: Optional[Stream] = None) -> None:
        check(lib().thork_memset(self.ptr, 0, self.nbytes, stream.handle if stream else None), "memset")


def to_device(arr: np.ndarray) -> DeviceArray:
    return DeviceArray.from_host(arr)


def empty(shape, dtype) -> DeviceArray:
    get_device()
    return DeviceArray(shape, dtype)


def copy_htod(d_ptr: int, arr: np.ndarray, stream: Optional[Stream] = None, sync: bool = True) -> None:
    check(lib().thork_memcpy_htod(d_ptr, arr.ctypes.data, arr.nbytes,
                                  stream.handle if stream else None, 1 if sync else 0), "memcpy HtoD")


def copy_dtoh(arr: np.ndarray, d_ptr: int, stream: Optional[Stream] = None, sync: bool = True) -> None:
    check(lib().thork_memcpy_dtoh(arr.ctypes.data, d_ptr, arr.nbytes,
                                  stream.handle if stream else None, 1 if sync else 0), "memcpy DtoH")


class _PinnedOwner:
    def __init__(self, ptr: int):
        self.ptr = ptr

    def __del__(self):
        try:
            lib().thork_host_free(self.ptr)
        except Exception:
            pass


def pinned_empty(shape, dtype) -> np.ndarray:
    """A NumPy array in page-locked host memory (fast DMA to/from the GPU).

    The allocation is released when the array and all views of it are gone.
    """
    get_device()
    dtype = np.dtype(dtype)
    n = int(np.prod(shape, dtype=np.int64)) * dtype.itemsize
    p = ctypes.c_void_p()
    check(lib().thork_host_alloc(max(n, 1), ctypes.byref(p)), "host alloc")
    raw = (ctypes.c_uint8 * max(n, 1)).from_address(p.value)
    raw._thork_owner = _PinnedOwner(p.value)  # freed with the buffer object
    return np.frombuffer(raw, dtype=np.uint8, count=n).view(dtype).reshape(shape)


def status_pointer() -> int:
    """Device address of the current device's kernel status word."""
    get_device()
    p = ctypes.c_void_p()
    check(lib().thork_status_pointer(ctypes.byref(p)), "status pointer")
    return p.value


def mem_info() -> Tuple[int, int]:
    """(free, total) bytes of device memory on the current device."""
    get_device()
    f, t = ctypes.c_size_t(0), ctypes.c_size_t(0)
    check(lib().thork_mem_info(ctypes.byref(f), ctypes.byref(t)), "mem info")
    return f.value, t.value


def noalloc_status(clear: bool = True, stream: Optional["Stream"] = None) -> int:
    """Status word of the allocation-free decode GEMM
    (``thork_skinny_gemm_bf16_noalloc``), which keeps its own word inside its
    static scratch array: non-zero after a bounded wait in one of its calls
    expired.  The word is sticky until read with ``clear``."""
    get_device()
    v = ctypes.c_uint(0)
    check(lib().thork_skinny_gemm_bf16_noalloc_status(
        ctypes.byref(v), 1 if clear else 0, stream.handle if stream else None), "no-alloc status")
    return v.value


# --------------------------------------------------------------------------
# compilation
# --------------------------------------------------------------------------
_NVRTC_LINE_RE = re.compile(r"(?:default_program|[A-Za-z0-9_./-]+\.cu)\((\d+)\)")


def rewrite_compile_error(log: str, source_map: Optional[Dict[int, Tuple[str, int]]]) -> str:
    """Prefix an NVRTC log with the Python locations of the generated lines
    it mentions (same header format as reference ``runtime.py:17-50``)."""
    if not source_map:
        return log
    seen = {}
    for m in _NVRTC_LINE_RE.finditer(log):
        ln = int(m.group(1))
        if ln in source_map and ln not in seen:
            seen[ln] = source_map[ln]
    if not seen:
        return log
    head = "\n".join(f"  generated line {ln} -> {f}:{l}" for ln, (f, l) in sorted(seen.items()))
    return f"Python source locations for reported generated lines:\n{head}\n\n{log}"


def cuda_include_dir() -> Optional[str]:
    for env in ("CUDA_HOME", "CUDA_PATH"):
        root = os.environ.get(env)
        if root and os.path.isdir(os.path.join(root, "include")):
            return os.path.join(root, "include")
    for cand in ("/usr/local/cuda/include", "/opt/cuda/include"):
        if os.path.isdir(cand):
            return cand
    return None


def _device_lib_digest() -> str:
    h = hashlib.sha256()
    for fn in sorted(os.listdir(DEVICE_INCLUDE)):
        with open(os.path.join(DEVICE_INCLUDE, fn), "rb") as f:
            h.update(fn.encode() + f.read())
    return h.hexdigest()


def _cache_dir() -> str:
    d = os.environ.get("THORK_CACHE_DIR") or os.path.join(
        os.path.expanduser("~"), ".cache", "thork_b200")
    os.makedirs(d, exist_ok=True)
    return d


def nvrtc_compile(source: str, *, source_map=None, extra_opts: Sequence[str] = (),
                  include_dirs: Sequence[str] = (), arch: str = ARCH,
                  name: str = "thork_kernel.cu", use_cache: bool = True) -> bytes:
    """Compile CUDA C++ to a cubin with NVRTC (no device needed).

    Raises ``RuntimeError("NVRTC compile failed: ...")`` with the log rewritten
    through ``source_map`` on error.
    """
    opts = ["-std=c++17", "-lineinfo", f"-I{DEVICE_INCLUDE}"]
    inc = cuda_include_dir()
    if inc:
        opts.append(f"-I{inc}")
    opts += [f"-I{d}" for d in include_dirs] + list(extra_opts)
    key = hashlib.sha256("\x00".join([source, arch, *opts, _device_lib_digest()]).encode()).hexdigest()
    path = os.path.join(_cache_dir(), f"{key}.cubin") if use_cache else None
    if path and os.path.exists(path):
        with open(path, "rb") as f:
            return f.read()
    c_opts = (ctypes.c_char_p * len(opts))(*[o.encode() for o in opts])
    cubin, size, log = ctypes.c_void_p(), ctypes.c_size_t(), ctypes.c_void_p()
    rc = lib().thork_nvrtc_compile(source.encode(), name.encode(), arch.encode(), c_opts, len(opts),
                                   ctypes.byref(cubin), ctypes.byref(size), ctypes.byref(log))
    log_text = ""
    if log.value:
        log_text = ctypes.string_at(log.value).decode("utf-8", errors="replace").rstrip("\x00 ")
        lib().thork_buffer_free(log.value)
    if rc != THORK_OK:
        msg = last_error()
        raise RuntimeError(
            f"NVRTC compile failed:\n{rewrite_compile_error(log_text, source_map)}\n({msg})"
            f"\n\nSource:\n{source}")
    data = ctypes.string_at(cubin.value, size.value)
    lib().thork_buffer_free(cubin.value)
    if path:
        tmp = f"{path}.{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    return data


class Module:
    """A cubin loaded into the current device's context."""

    def __init__(self, cubin: bytes):
        get_device()
        self._image = ctypes.create_string_buffer(cubin, len(cubin))
        h = ctypes.c_void_p()
        check(lib().thork_module_load(self._image, ctypes.byref(h)), "module load")
        self.handle = h.value
        self._funcs: Dict[str, int] = {}

    def function(self, name: str) -> int:
        if name not in self._funcs:
            h = ctypes.c_void_p()
            check(lib().thork_module_get_function(self.handle, name.encode(), ctypes.byref(h)),
                  f"get function {name}")
            self._funcs[name] = h.value
        return self._funcs[name]


def compile_source(source: str, *, source_map=None, extra_opts: Sequence[str] = (),
                   include_dirs: Sequence[str] = ()) -> Module:
    """NVRTC -> cubin (sm_100a) -> loaded module (reference ``runtime.py:373-421``)."""
    return Module(nvrtc_compile(source, source_map=source_map, extra_opts=extra_opts,
                                include_dirs=include_dirs))


def _nvcc_path() -> str:
    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH") or "/usr/local/cuda"
    cand = os.path.join(home, "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    import shutil
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def nvcc_compile(source: str, *, source_map=None, extra_opts: Optional[Sequence[str]] = None,
                 include_dirs: Optional[Sequence[str]] = None,
                 defines: Optional[Sequence[str]] = None) -> bytes:
    """nvcc -> sm_100a cubin, for sources that need headers NVRTC cannot
    reach.  Raises ``RuntimeError("nvcc compile failed: ...")`` with the log
    rewritten to Python source locations."""
    import subprocess
    import tempfile
    with tempfile.TemporaryDirectory(prefix="thork_b200_") as tmp:
        src = os.path.join(tmp, "kernel.cu")
        out = os.path.join(tmp, "kernel.cubin")
        with open(src, "w") as f:
            f.write(source)
        cmd = [_nvcc_path(), "--cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17",
               "-lineinfo", "-I", os.path.join(PKG_DIR, "csrc", "device")]
        for d in include_dirs or ():
            cmd += ["-I", d]
        for d in defines or ():
            cmd.append(d if d.startswith("-D") else "-D" + d)
        cmd += list(extra_opts or ()) + [src, "-o", out]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            log = (r.stdout + r.stderr).replace(src, "<thork kernel>")
            raise RuntimeError(f"nvcc compile failed:\n{rewrite_compile_error(log, source_map)}")
        with open(out, "rb") as f:
            return f.read()


def compile_source_with_nvcc(source: str, *, source_map=None,
                             extra_opts: Optional[Sequence[str]] = None,
                             include_dirs: Optional[Sequence[str]] = None,
                             defines: Optional[Sequence[str]] = None) -> Module:
    """nvcc -> cubin (sm_100a) -> loaded module (reference ``runtime.py:312-338``)."""
    return Module(nvcc_compile(source, source_map=source_map, extra_opts=extra_opts,
                               include_dirs=include_dirs, defines=defines))


def compile_source_to_shared_lib(source: str, **kwargs):
    """The reference builds ThunderKittens kernels into host shared libraries
    with generated launchers (``runtime.py:341-371``).  Tile kernels here are
    NVRTC cubins launched through ``thork_launch``, so there is no host
    launcher to build."""
    raise NotImplementedError(
        "compile_source_to_shared_lib: tile kernels compile to NVRTC cubins here and launch "
        "through thork_launch; use compile_source() or @tk.jit")


def dispatch_tk(lib, kernel_name, params, user_args, grid_size, block_size, shared_mem_bytes,
                stream=0):
    """Reference ``runtime.py:534-612`` launches ThunderKittens kernels through
    their generated host launcher; ``dispatch`` launches every kernel here."""
    raise NotImplementedError(
        "dispatch_tk: tile kernels launch through runtime.dispatch (no generated host launcher)")


def kittens_include_dirs() -> List[str]:
    """Include directories of the tile library the tile kernels compile
    against (reference ``runtime.py:121-136`` returns ThunderKittens')."""
    return [os.path.join(PKG_DIR, "csrc", "device")]


def kittens_sm_define_for_cap(cap: str) -> str:
    """Architecture define for a compute capability string such as
    ``"100"`` or ``"100a"`` (reference ``runtime.py:139-154``), for code that
    passes it on to its own builds; the tile library itself is sm_100a."""
    digits = cap.rstrip("a")
    major = int(digits[:-1]) if len(digits) > 2 else int(digits[0])
    if major >= 12:
        return "KITTENS_SM120"
    if major >= 10:
        return "KITTENS_SM100"
    return "KITTENS_SM90" if major == 9 else "KITTENS_SM80"


def kittens_sm_define() -> str:
    return kittens_sm_define_for_cap(get_compute_capability())


def set_max_dynamic_shared_size(func: int) -> None:
    """Opt ``func`` into the device's dynamic shared memory budget minus the
    1 KiB reserve (reference ``runtime.py:189-200``)."""
    check(lib().thork_function_set_max_dynamic_smem(func, max_dynamic_shared_size()),
          "set max dynamic shared size")


def get_function(module: Module, name: str) -> int:
    return module.function(name)


def launch(func: int, grid, block, args: List[ctypes._SimpleCData], *, smem: int = 0,
           stream: Optional[Stream] = None, cluster=None) -> None:
    """Launch with kernel-parameter storage ``args`` (ctypes objects)."""
    n = len(args)
    ptrs = (ctypes.c_void_p * max(n, 1))(*[ctypes.cast(ctypes.pointer(a), ctypes.c_void_p) for a in args])
    g = (ctypes.c_uint * 3)(*[int(x) for x in grid])
    b = (ctypes.c_uint * 3)(*[int(x) for x in block])
    c = (ctypes.c_uint * 3)(*[int(x) for x in cluster]) if cluster else None
    check(lib().thork_launch(func, g, b, c, int(smem), stream.handle if stream else None, ptrs),
          "launch")


# --------------------------------------------------------------------------
# argument validation and dispatch (reference runtime.py:431-700)
# --------------------------------------------------------------------------
def _expect_pointer_arg(arr, param: ir.Param):
    if isinstance(arr, DeviceArray):
        if not dt.storage_compatible(arr.dtype, param.dtype):
            raise TypeError(
                f"Argument for pointer parameter '{param.name}' has dtype {arr.dtype}, "
                f"expected {param.dtype.name}")
        return arr
    if not isinstance(arr, np.ndarray):
        raise TypeError(
            f"Argument for pointer parameter '{param.name}' must be a numpy array, "
            f"got {type(arr).__name__}")
    if not dt.storage_compatible(arr.dtype, param.dtype):
        actual = dt.from_numpy(arr.dtype)  # raises TypeError for unmapped dtypes
        raise TypeError(
            f"Argument for pointer parameter '{param.name}' has dtype {actual.name}, "
            f"expected {param.dtype.name}")
    if not arr.flags["C_CONTIGUOUS"]:
        raise ValueError(f"Argument for pointer parameter '{param.name}' must be C-contiguous")
    return arr


def _expect_kittens_arg(arr, param: ir.Param):
    if not isinstance(arr, (np.ndarray, DeviceArray)):
        raise TypeError(
            f"Argument for kittens.Global parameter '{param.name}' must be a numpy array, "
            f"got {type(arr).__name__}")
    if arr.ndim != 2:
        raise TypeError(
            f"kittens.Global parameter '{param.name}' requires a 2-D numpy array, got shape "
            f"{arr.shape}")
    if arr.dtype.itemsize != param.dtype.nbytes:
        raise TypeError(
            f"Argument for kittens.Global parameter '{param.name}' has {arr.dtype.itemsize}-byte "
            f"elements; expected {param.dtype.nbytes} to match {param.dtype.name}")
    if isinstance(arr, np.ndarray) and not arr.flags["C_CONTIGUOUS"]:
        raise ValueError(
            f"Argument for kittens.Global parameter '{param.name}' must be C-contiguous")
    return arr


_SCALAR_CTYPES = {
    "float32": ctypes.c_float, "float16": ctypes.c_uint16, "int32": ctypes.c_int32,
    "uint32": ctypes.c_uint32, "int64": ctypes.c_int64, "uint64": ctypes.c_uint64,
    "bool": ctypes.c_int32,
}
_VEC_CTYPES = {"uint2": (ctypes.c_uint32, 2), "uint3": (ctypes.c_uint32, 3),
               "int2": (ctypes.c_int32, 2), "int3": (ctypes.c_int32, 3)}


def _scalar_storage(value, param: ir.Param):
    if param.vec_size > 1:
        ct, n = _VEC_CTYPES[param.cuda_name]
        vals = list(value)
        if len(vals) != n:
            raise TypeError(f"Argument for '{param.name}' must have {n} components")
        return (ct * n)(*[int(v) for v in vals])
    ct = _SCALAR_CTYPES.get(param.dtype.name)
    if ct is None:
        raise TypeError(f"No ctypes mapping for constant scalar dtype {param.dtype.name}")
    if param.dtype.name == "float16":
        return ct(int(np.asarray(value, np.float16).view(np.uint16)))
    if param.dtype.is_float:
        return ct(float(value))
    return ct(int(np.asarray(value).astype(np.int64)) & ((1 << (8 * ctypes.sizeof(ct))) - 1)
              if not param.dtype.is_signed else int(value))


GL_BYTES = 192  # sizeof(thork::tk::gl<...>): tensor map (128) + ptr + rows + cols, 64-aligned


def tile_swizzle_bytes(cols: int, elem: int) -> int:
    """Swizzle width of a row-major shared tile whose rows are cols*elem bytes
    (the same rule thork_tk.cuh applies)."""
    rb = cols * elem
    for sw in (128, 64, 32):
        if rb % sw == 0:
            return sw
    return 0


def pack_global(ptr: int, rows: int, cols: int, param: ir.Param):
    """Kernel-parameter bytes of ``thork::tk::gl<T, R, C>``."""
    buf = (ctypes.c_uint8 * (GL_BYTES + 64))()
    base = ctypes.addressof(buf)
    off = (-base) % 64
    tmap_addr = base + off
    if param.tile_shape is not None:
        tr, tc = param.tile_shape
        elem = param.dtype.nbytes
        sw = tile_swizzle_bytes(tc, elem)
        box_cols = sw // elem if sw else tc
        box_rows = min(tr, 256)
        code = DT_CODE.get(param.dtype.name, 0)
        check(lib().thork_tensor_map_2d(tmap_addr, code, ptr, rows, cols, cols * elem, box_rows,
                                        box_cols, sw), f"tensor map for '{param.name}'")
    struct.pack_into("<QQQ", buf, off + 128, int(ptr), int(rows), int(cols))
    out = (ctypes.c_uint8 * GL_BYTES).from_buffer_copy(bytes(buf)[off:off + GL_BYTES])
    return out


def dispatch(func: int, params: Sequence[ir.Param], user_args: Sequence, grid_size, block_size,
             shared_mem_bytes: int = 0, stream: int = 0, *, uses_status: bool = False,
             name: str = "kernel", cluster=None) -> None:
    """Copy NumPy arguments in, launch, synchronise, copy written buffers back.

    DeviceArray arguments are used in place (no copies).  Only parameters the
    trace marked ``written`` are copied back, into the caller's arrays.
    """
    get_device()
    bindable = [p for p in params if p.bindable]
    if len(user_args) != len(bindable):
        raise TypeError(
            f"Kernel expected {len(bindable)} arguments (pointer + constant + kittens_global "
            f"params), got {len(user_args)}")
    s = _dispatch_stream()
    storage = []
    copies_back = []
    owned: List[DeviceBuffer] = []
    try:
        for p, a in zip(bindable, user_args):
            if p.kind in ("pointer", "kittens_global"):
                arr = _expect_pointer_arg(a, p) if p.kind == "pointer" else _expect_kittens_arg(a, p)
                if isinstance(arr, DeviceArray):
                    ptr = arr.ptr
                else:
                    buf = DeviceBuffer(arr.nbytes)
                    owned.append(buf)
                    ptr = buf.ptr
                    copy_htod(ptr, arr, s, sync=False)
                    if p.written:
                        copies_back.append((arr, ptr))
                if p.kind == "pointer":
                    storage.append(ctypes.c_void_p(ptr))
                else:
                    storage.append(pack_global(ptr, arr.shape[0], arr.shape[1], p))
            else:
                storage.append(_scalar_storage(a, p))
        if uses_status:
            storage.append(ctypes.c_void_p(status_pointer()))
        launch(func, grid_size, block_size, storage, smem=shared_mem_bytes, stream=s,
               cluster=cluster)
        for arr, ptr in copies_back:
            copy_dtoh(arr, ptr, s, sync=False)
        s.synchronize()
        if uses_status:
            check_kernel_status(name)
    finally:
        for b in owned:
            b.free()


class PreparedLaunch:
    """A traced kernel with its arguments packed once, for repeated
    asynchronous launches on device-resident data (for example back-to-back
    launches timed with events, or a launch sequence without Python argument
    handling in between).

    Every pointer / global argument must be a ``DeviceArray`` (nothing is
    copied in or back).  ``launch(stream)`` queues the kernel and returns at
    once; a kernel with bounded waits reports to the device status word, read
    with ``kernel_status()`` after synchronising.  No reference counterpart:
    the reference's launches always copy and synchronise
    (``runtime.py:656-700``)."""

    def __init__(self, func: int, params: Sequence[ir.Param], user_args: Sequence, grid_size,
                 block_size, shared_mem_bytes: int = 0, *, uses_status: bool = False,
                 cluster=None):
        get_device()
        bindable = [p for p in params if p.bindable]
        if len(user_args) != len(bindable):
            raise TypeError(
                f"Kernel expected {len(bindable)} arguments (pointer + constant + kittens_global "
                f"params), got {len(user_args)}")
        storage = []
        for p, a in zip(bindable, user_args):
            if p.kind in ("pointer", "kittens_global"):
                if not isinstance(a, DeviceArray):
                    raise TypeError(f"prepared launches take DeviceArray arguments; parameter "
                                    f"'{p.name}' got {type(a).__name__}")
                arr = _expect_pointer_arg(a, p) if p.kind == "pointer" else _expect_kittens_arg(a, p)
                storage.append(ctypes.c_void_p(arr.ptr) if p.kind == "pointer"
                               else pack_global(arr.ptr, arr.shape[0], arr.shape[1], p))
            else:
                storage.append(_scalar_storage(a, p))
        if uses_status:
            storage.append(ctypes.c_void_p(status_pointer()))
        self._storage = storage  # keeps the argument bytes alive
        n = len(storage)
        self._ptrs = (ctypes.c_void_p * max(n, 1))(
            *[ctypes.cast(ctypes.pointer(a), ctypes.c_void_p) for a in storage])
        self._grid = (ctypes.c_uint * 3)(*[int(x) for x in grid_size])
        self._block = (ctypes.c_uint * 3)(*[int(x) for x in block_size])
        self._cluster = (ctypes.c_uint * 3)(*[int(x) for x in cluster]) if cluster else None
        self._func = func
        self._smem = int(shared_mem_bytes)

    def launch(self, stream: Optional[Stream] = None) -> None:
        check(lib().thork_launch(self._func, self._grid, self._block, self._cluster, self._smem,
                                 stream.handle if stream else None, self._ptrs), "launch")
