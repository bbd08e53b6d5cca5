"""thork_b200.kittens — tile operations in the ThunderKittens vocabulary,
lowered to this package's own sm_100a device library (``thork_tk.cuh``).

Front end of the reference's ``src/thork/kittens.py``: the same names and
argument conventions (``kittens.py:240-857``); the generated code calls
``thork::tk::`` functions written for B200 (TMA tensor maps, mbarriers,
tcgen05 + TMEM) instead of ThunderKittens templates.
"""

from . import dtypes as dt
from . import ir
from .tracer import KernelBuilder
from .types import KittensGlobal as Global  # noqa: F401  (re-export)

_ELEM = {"float32": "float", "float16": "__half", "bfloat16": "__nv_bfloat16",
         "float8_e4m3": "unsigned char", "int32": "int", "uint32": "unsigned int"}


def elem_ctype(d: dt.Dtype) -> str:
    if d.name not in _ELEM:
        raise TypeError(f"thork dtype {d.name} has no tile-library equivalent")
    return _ELEM[d.name]


def mark_kittens(b: KernelBuilder) -> None:
    """Flag a kernel as using the tile library (adds its include)."""
    if not b.uses_kittens:
        b.uses_kittens = True
        b.add_include("thork_tk.cuh", system=False)


class _Handle:
    __slots__ = ("_expr", "_dtype", "_builder", "_stype")

    def __init__(self, expr: ir.Expr, dtype: dt.Dtype, builder: KernelBuilder):
        self._expr = expr
        self._dtype = dtype
        self._builder = builder
        self._stype = None


class GlobalHandle(_Handle):
    """A ``kittens.Global`` kernel parameter."""

    __slots__ = ("_param_name", "_tile_shape")

    def __init__(self, expr: ir.Name, dtype: dt.Dtype, builder: KernelBuilder, tile_shape=None):
        super().__init__(expr, dtype, builder)
        self._param_name = expr.name
        self._tile_shape = tile_shape


KittensGlobalTracer = GlobalHandle


def finalize(b: KernelBuilder) -> None:
    """Hook run after tracing a tile kernel (shared-memory sizing)."""
    b.dynamic_smem = getattr(b, "dynamic_smem", 0)
