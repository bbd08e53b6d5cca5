"""Element types of thork_b200 kernels (``tk.dt``).

Mirrors the reference's dtype table (``src/thork/dtypes.py:18-25``) and adds
the two types the B200 tile path needs: ``bfloat16`` gets a NumPy mapping
(through ml_dtypes, or raw ``uint16`` storage), and ``float8_e4m3`` is new
(the reference has no FP8 type).
"""

from dataclasses import dataclass
from typing import Optional

import numpy as np

try:  # ml_dtypes provides NumPy scalar types for bf16 and e4m3
    import ml_dtypes as _ml
except ImportError:  # pragma: no cover - ml_dtypes ships with the image
    _ml = None


@dataclass(frozen=True)
class Dtype:
    """A kernel element type: its name, CUDA spelling and size in bytes."""

    name: str
    cuda: str
    nbytes: int
    is_float: bool = False
    is_signed: bool = True

    def __repr__(self) -> str:
        return f"dt.{self.name}"

    @property
    def numpy(self) -> Optional[np.dtype]:
        """The NumPy dtype that stores this type natively, if any."""
        return _NATIVE_NUMPY.get(self.name)


float32 = Dtype("float32", "float", 4, is_float=True)
float16 = Dtype("float16", "__half", 2, is_float=True)
bfloat16 = Dtype("bfloat16", "__nv_bfloat16", 2, is_float=True)
float8_e4m3 = Dtype("float8_e4m3", "__nv_fp8_e4m3", 1, is_float=True)
int32 = Dtype("int32", "int", 4)
uint32 = Dtype("uint32", "unsigned int", 4, is_signed=False)
int64 = Dtype("int64", "long long", 8)
uint64 = Dtype("uint64", "unsigned long long", 8, is_signed=False)
bool_ = Dtype("bool", "bool", 1, is_signed=False)

ALL = (float32, float16, bfloat16, float8_e4m3, int32, uint32, int64, uint64, bool_)

_NATIVE_NUMPY = {
    "float32": np.dtype(np.float32),
    "float16": np.dtype(np.float16),
    "int32": np.dtype(np.int32),
    "uint32": np.dtype(np.uint32),
    "int64": np.dtype(np.int64),
    "uint64": np.dtype(np.uint64),
    "bool": np.dtype(np.bool_),
}
if _ml is not None:
    _NATIVE_NUMPY["bfloat16"] = np.dtype(_ml.bfloat16)
    _NATIVE_NUMPY["float8_e4m3"] = np.dtype(_ml.float8_e4m3fn)

_FROM_NUMPY = {v: globals()[k if k != "bool" else "bool_"] for k, v in _NATIVE_NUMPY.items()}


def from_numpy(np_dtype) -> Dtype:
    """Map a NumPy dtype to its thork dtype (``TypeError`` when none)."""
    key = np.dtype(np_dtype)
    if key not in _FROM_NUMPY:
        raise TypeError(f"No thork dtype for numpy dtype {np_dtype}")
    return _FROM_NUMPY[key]


def storage_compatible(arr_dtype, d: Dtype) -> bool:
    """True when an array of ``arr_dtype`` may back a ``d`` buffer.

    Exact NumPy matches always qualify.  For the 16-bit and 8-bit float types
    raw unsigned storage of the same width (``uint16`` for bf16, ``uint8`` for
    e4m3) is accepted too, the convention the reference's tile tests use for
    bf16 (``tests/test_kittens.py:20-28``).
    """
    arr_dtype = np.dtype(arr_dtype)
    if d.numpy is not None and arr_dtype == d.numpy:
        return True
    if d.name == "bfloat16":
        return arr_dtype == np.dtype(np.uint16)
    if d.name == "float8_e4m3":
        return arr_dtype == np.dtype(np.uint8)
    return False


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round a float array to bf16 (nearest-even) and return the raw
    ``uint16`` bit patterns, the storage the tile kernels consume."""
    if _ml is None:  # pragma: no cover
        raise RuntimeError("ml_dtypes is required for bf16 conversion")
    return np.asarray(x, np.float32).astype(_ml.bfloat16).view(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    """Widen raw bf16 bit patterns (``uint16``) to float32."""
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def quantize_e4m3(x: np.ndarray):
    """Per-tensor FP8 quantisation: ``scale = amax / 448`` and the e4m3fn bytes
    of ``x / scale`` (nearest-even).  Returns ``(uint8 array, float scale)``."""
    if _ml is None:  # pragma: no cover
        raise RuntimeError("ml_dtypes is required for e4m3 conversion")
    x = np.asarray(x, np.float32)
    amax = float(np.max(np.abs(x))) if x.size else 0.0
    scale = np.float32(amax / 448.0) if amax > 0 else np.float32(1.0)
    q = np.clip(x / scale, -448.0, 448.0).astype(_ml.float8_e4m3fn).view(np.uint8)
    return q, float(scale)
