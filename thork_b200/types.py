"""Parameter annotations of ``@tk.jit`` kernels.

The annotation vocabulary is the reference's (``src/thork/types.py``):

* thread-attribute markers ``BlockIdx, ThreadIdx, BlockDim, GridDim,
  WarpSize, LaneId, WarpId`` (``types.py:7-51``);
* ``DevicePointer[dtype]`` -> a ``T *`` kernel argument bound to a NumPy
  array (``types.py:107-116``);
* ``kittens.Global[dtype]`` / ``kittens.Global[dtype, (R, C)]`` -> a 2-D
  tile-addressed global, optionally with a TMA box of R x C
  (``types.py:119-164``);
* ``Uint, Uint2, Uint3, Int, Int2, Int3``: subscripted with a marker they
  become kernel-entry built-ins, bare they are by-value scalars
  (``types.py:167-195``).
"""

from dataclasses import dataclass
from typing import Optional, Tuple, Type

from . import dtypes as dt


class ThreadAttribute:
    """Marker for a value synthesised at kernel entry from a CUDA built-in.

    ``cuda_expr`` names the built-in; vector built-ins (``blockIdx`` ...)
    expose ``.x/.y/.z`` while scalar ones are complete expressions.
    """

    cuda_expr: str = ""
    vector: bool = True


class BlockIdx(ThreadAttribute):
    cuda_expr = "blockIdx"


class ThreadIdx(ThreadAttribute):
    cuda_expr = "threadIdx"


class BlockDim(ThreadAttribute):
    cuda_expr = "blockDim"


class GridDim(ThreadAttribute):
    cuda_expr = "gridDim"


class WarpSize(ThreadAttribute):
    cuda_expr = "warpSize"
    vector = False


class LaneId(ThreadAttribute):
    """Lane within the warp (``threadIdx.x & 31`` for 1-D blocks)."""

    cuda_expr = "(threadIdx.x & 0x1f)"
    vector = False


class WarpId(ThreadAttribute):
    """Warp within the block (``threadIdx.x >> 5`` for 1-D blocks)."""

    cuda_expr = "(threadIdx.x >> 5)"
    vector = False


@dataclass(frozen=True)
class DevicePointerSpec:
    """``T *name``: bound to a C-contiguous NumPy array of matching dtype."""

    dtype: dt.Dtype


@dataclass(frozen=True)
class KittensGlobalSpec:
    """A 2-D row-major global addressed in tiles.

    ``tile_shape`` (rows, cols) is the TMA box; it is required by the
    ``kittens.tma.*`` operations and fixes the unit of tile coordinates.
    """

    dtype: dt.Dtype
    tile_shape: Optional[Tuple[int, int]] = None


@dataclass(frozen=True)
class ScalarParamSpec:
    """A scalar or 2/3-vector parameter.

    With ``attribute`` set it is synthesised from a CUDA built-in; without it,
    the host passes it by value.
    """

    dtype: dt.Dtype
    cuda_name: str
    vec_size: int = 1
    attribute: Optional[Type[ThreadAttribute]] = None


class _ScalarTypeBase:
    """Base of the bare scalar annotation classes (``tk.Uint`` ...)."""

    _dtype: dt.Dtype
    _cuda_name: str
    _vec_size: int = 1


class DevicePointer:
    """``tk.DevicePointer[dtype]``."""

    def __class_getitem__(cls, dtype) -> DevicePointerSpec:
        if not isinstance(dtype, dt.Dtype):
            raise TypeError(f"DevicePointer[...] expects a thork dtype, got {dtype!r}")
        return DevicePointerSpec(dtype=dtype)


class KittensGlobal:
    """``tk.kittens.Global[dtype]`` or ``tk.kittens.Global[dtype, (R, C)]``."""

    def __class_getitem__(cls, args) -> KittensGlobalSpec:
        items = args if isinstance(args, tuple) else (args,)
        if not items:
            raise TypeError("kittens.Global[...] requires at least a dtype")
        dtype, extras = items[0], items[1:]
        if not isinstance(dtype, dt.Dtype):
            raise TypeError(
                "kittens.Global[...] expects a thork dtype as the first argument, "
                f"got {dtype!r}"
            )
        if len(extras) > 1:
            raise TypeError(
                "kittens.Global[dtype, (R, C)] accepts at most one tile shape; "
                f"got {len(extras)} extras"
            )
        shape = None
        if extras:
            shape = extras[0]
            ok = (isinstance(shape, tuple) and len(shape) == 2
                  and all(isinstance(v, int) and not isinstance(v, bool) and v > 0 for v in shape))
            if not ok:
                raise TypeError(
                    "kittens.Global tile shape must be a (rows, cols) tuple of positive "
                    f"ints, got {shape!r}"
                )
        return KittensGlobalSpec(dtype=dtype, tile_shape=shape)


def _scalar_type(dtype: dt.Dtype, cuda_name: str, vec_size: int):
    def class_getitem(cls, attribute):
        if not (isinstance(attribute, type) and issubclass(attribute, ThreadAttribute)):
            raise TypeError(
                f"{cuda_name}[...] expects a ThreadAttribute subclass, got {attribute!r}"
            )
        return ScalarParamSpec(dtype=dtype, cuda_name=cuda_name, vec_size=vec_size,
                               attribute=attribute)

    name = {"unsigned int": "Uint", "int": "Int"}.get(cuda_name, cuda_name.capitalize())
    return type(name, (_ScalarTypeBase,), {
        "_dtype": dtype,
        "_cuda_name": cuda_name,
        "_vec_size": vec_size,
        "__class_getitem__": classmethod(class_getitem),
    })


Uint = _scalar_type(dt.uint32, "unsigned int", 1)
Uint2 = _scalar_type(dt.uint32, "uint2", 2)
Uint3 = _scalar_type(dt.uint32, "uint3", 3)
Int = _scalar_type(dt.int32, "int", 1)
Int2 = _scalar_type(dt.int32, "int2", 2)
Int3 = _scalar_type(dt.int32, "int3", 3)


def spec_from_annotation(ann, kernel_name: str, param_name: str):
    """Normalise an annotation to a DevicePointerSpec / ScalarParamSpec /
    KittensGlobalSpec (reference ``jit.py:12-38``)."""
    if isinstance(ann, (DevicePointerSpec, ScalarParamSpec, KittensGlobalSpec)):
        return ann
    if isinstance(ann, type) and issubclass(ann, _ScalarTypeBase):
        return ScalarParamSpec(dtype=ann._dtype, cuda_name=ann._cuda_name,
                               vec_size=ann._vec_size, attribute=None)
    raise TypeError(
        f"Kernel '{kernel_name}': parameter '{param_name}' has unsupported annotation "
        f"{ann!r}. Expected tk.DevicePointer[...], tk.Uint[...] or tk.kittens.Global[...]."
    )
