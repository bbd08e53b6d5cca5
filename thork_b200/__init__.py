"""thork_b200 — a B200-native (sm_100a) codegen and runtime for the thork
tracing DSL.

Drop-in for ``import thork as tk`` (reference ``src/thork/__init__.py``)::

    import thork_b200 as tk

    @tk.jit
    def add(out: tk.DevicePointer[tk.dt.float32], a: tk.DevicePointer[tk.dt.float32],
            b: tk.DevicePointer[tk.dt.float32], bid: tk.Uint[tk.BlockIdx],
            tid: tk.Uint[tk.ThreadIdx], bdm: tk.Uint[tk.BlockDim]):
        i = bid * bdm + tid
        out[i] = a[i] + b[i]

    add[(n // 128, 1, 1), (128, 1, 1)](C, A, B)

Kernels compile through NVRTC to sm_100a cubins and launch through
``libthork_rt.so``; the library kernels (``tk.kernels``) are hand-written
tcgen05/TMA CUDA compiled ahead of time.  There is no CPU fallback.
"""

from . import dtypes as dt
from . import kernels
from . import kittens
from . import runtime
from .jit import BoundKernel, JittedKernel, jit
from .tracer import (
    DeviceFn, abs, acos, all_sync, any_sync, asin, atan, atan2, atomic_add, atomic_and,
    atomic_cas, atomic_exch, atomic_max, atomic_min, atomic_or, atomic_sub, atomic_xor,
    ballot_sync, break_, cast, ceil, continue_, cos, cosh, device_fn, exp, exp2, fabs,
    fast_cos, fast_exp, fast_log, fast_log10, fast_log2, fast_pow, fast_rsqrt, fast_sin,
    fast_sqrt, fast_tan, floor, fma, fmax, fmin, fmod, if_, local, log, log10, log2, max, min,
    pow, range, round, rsqrt, shared, shfl_down_sync, shfl_sync, shfl_up_sync, shfl_xor_sync,
    sin, sinh, sqrt, syncthreads, syncwarp, tan, tanh, trunc, warp_sum, while_,
)
from .types import (
    BlockDim, BlockIdx, DevicePointer, GridDim, Int, Int2, Int3, LaneId, ScalarParamSpec,
    ThreadAttribute, ThreadIdx, Uint, Uint2, Uint3, WarpId, WarpSize,
)

__all__ = [
    "dt", "kernels", "kittens", "runtime", "jit", "JittedKernel", "BoundKernel",
    "local", "range", "if_", "while_", "break_", "continue_", "device_fn", "DeviceFn",
    "shared", "syncthreads", "syncwarp", "cast",
    "exp", "exp2", "log", "log2", "log10", "sqrt", "rsqrt",
    "sin", "cos", "tan", "asin", "acos", "atan", "atan2", "sinh", "cosh", "tanh",
    "floor", "ceil", "round", "trunc", "fabs", "abs",
    "pow", "fmod", "fmin", "fmax", "min", "max", "fma",
    "fast_exp", "fast_log", "fast_log2", "fast_log10", "fast_sqrt", "fast_rsqrt",
    "fast_sin", "fast_cos", "fast_tan", "fast_pow",
    "shfl_sync", "shfl_up_sync", "shfl_down_sync", "shfl_xor_sync",
    "ballot_sync", "all_sync", "any_sync", "warp_sum",
    "atomic_add", "atomic_sub", "atomic_and", "atomic_or", "atomic_xor",
    "atomic_min", "atomic_max", "atomic_exch", "atomic_cas",
    "DevicePointer", "ScalarParamSpec", "Uint", "Uint2", "Uint3", "Int", "Int2", "Int3",
    "ThreadAttribute", "BlockIdx", "ThreadIdx", "BlockDim", "GridDim",
    "WarpSize", "LaneId", "WarpId",
]
