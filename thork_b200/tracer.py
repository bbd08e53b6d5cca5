"""Tracing front end: Python values that record CUDA IR while a ``@tk.jit``
function runs once.

Same user-facing vocabulary as the reference tracer (``src/thork/tracer.py``):
scalar arithmetic through operator overloads (``tracer.py:207-292``), pointer
loads/stores that mark written buffers (``tracer.py:295-319``), ``.x/.y/.z``
vectors (``322-346``), ``tk.local`` mutable locals (``349-426``),
``tk.range`` loops (``429-480``), ``tk.shared`` arrays (``483-551``),
barriers, warp shuffles and ``warp_sum`` (``554-691``), ``if_/else_/while_/
break_/continue_`` (``694-823``), math intrinsics and ``cast`` (``831-897``),
atomics (``905-961``) and ``device_fn`` (``969-1096``).

Implementation notes: statements go to the innermost open block of a
``KernelBuilder`` block stack; each statement records the user's
(file, line), found by walking the stack to the first frame outside this
package.
"""

import builtins
import contextvars
import inspect
import os
import sys
from typing import Callable, Dict, List, Optional

from . import dtypes as dt
from . import ir
from .types import DevicePointerSpec

_PKG_DIR = os.path.dirname(os.path.abspath(__file__)) + os.sep


_stype_hooks: dict = {}


def register_stype_hooks(**hooks) -> None:
    """Registration point for a verification side-car's type-combination
    hooks (keys ``binop``, ``unary``, ``math``, ``scalar``, ``local_init``;
    reference ``tracer.py:144-154``).  The hooks are kept; tracing does not
    consult them, since the verifier they serve is not part of this
    package."""
    unknown = set(hooks) - {"binop", "unary", "math", "scalar", "local_init"}
    if unknown:
        raise TypeError(f"register_stype_hooks: unknown hook(s) {sorted(unknown)}")
    _stype_hooks.update(hooks)


def user_location():
    """(filename, line) of the innermost frame outside the thork_b200 package."""
    f = sys._getframe(1)
    while f is not None:
        if not f.f_code.co_filename.startswith(_PKG_DIR):
            return (f.f_code.co_filename, f.f_lineno)
        f = f.f_back
    return None


_active: contextvars.ContextVar = contextvars.ContextVar("thork_b200_builder", default=None)


def current_builder() -> "KernelBuilder":
    b = _active.get()
    if b is None:
        raise RuntimeError("thork operations may only be used inside a @tk.jit-decorated kernel")
    return b


class KernelBuilder:
    """Accumulates the parameters, statements and requirements of one kernel
    (or device function) during tracing."""

    def __init__(self, name: str):
        self.name = name
        self.params: List[ir.Param] = []
        self._blocks: List[List[ir.Stmt]] = [[]]
        self.includes: List[tuple] = [("cuda_fp16.h", True), ("cuda_bf16.h", True)]
        self.uses_kittens = False      # any tile op: include the tile library
        self.uses_tma = False          # TMA ops: globals carry tensor maps
        self.uses_status = False       # bounded waits: hidden status pointer
        self.device_functions: List["DeviceFn"] = []
        self._counters: Dict[str, int] = {}
        # text emitted right after the attribute locals / before the closing
        # brace (tile-library set-up and teardown)
        self.prologue: List[str] = []
        self.epilogue: List[str] = []

    # -- statements
    @property
    def stmts(self) -> List[ir.Stmt]:
        return self._blocks[0]

    def add_stmt(self, stmt: ir.Stmt) -> None:
        if getattr(stmt, "loc", None) is None:
            stmt.loc = user_location()
        self._blocks[-1].append(stmt)

    def open_block(self) -> None:
        self._blocks.append([])

    def close_block(self) -> List[ir.Stmt]:
        return self._blocks.pop()

    def last_stmt(self) -> Optional[ir.Stmt]:
        blk = self._blocks[-1]
        return blk[-1] if blk else None

    # -- names / params
    def fresh_name(self, prefix: str = "v") -> str:
        n = self._counters.get(prefix, 0)
        self._counters[prefix] = n + 1
        return f"{prefix}{n}"

    def find_param(self, name: str) -> Optional[ir.Param]:
        for p in self.params:
            if p.name == name:
                return p
        return None

    def mark_written(self, expr: ir.Expr, kinds=("pointer",)) -> None:
        if isinstance(expr, ir.Name):
            p = self.find_param(expr.name)
            if p is not None and p.kind in kinds:
                p.written = True

    def add_include(self, path: str, system: bool = True) -> None:
        if (path, system) not in self.includes:
            self.includes.append((path, system))

    def add_device_fn(self, df: "DeviceFn") -> None:
        df._ensure_traced()
        for dep in df._deps:
            self.add_device_fn(dep)
        if any(d._name == df._name for d in self.device_functions):
            return
        self.device_functions.append(df)
        for inc in df._includes:
            self.add_include(*inc)


# --------------------------------------------------------------------------
# values
# --------------------------------------------------------------------------
def to_expr(v) -> ir.Expr:
    if isinstance(v, Value):
        return v._expr
    if isinstance(v, Vector):
        raise TypeError("Cannot use a vector value as a scalar — access a field like .x first")
    if isinstance(v, Pointer):
        raise TypeError("Cannot use a pointer as a scalar value — index it with ptr[i]")
    if isinstance(v, (bool, int, float)):
        return ir.Lit(v)
    raise TypeError(f"Cannot convert {v!r} (type {type(v).__name__}) to a thork expression")


def _promote(a: Optional[dt.Dtype], b) -> Optional[dt.Dtype]:
    bd = b._dtype if isinstance(b, Value) else None
    if a is not None and bd is not None:
        if a.is_float or bd.is_float:
            return a if a.is_float else bd
        return a
    return a or bd


class Value:
    """A traced scalar expression."""

    __slots__ = ("_expr", "_dtype", "_stype")

    def __init__(self, expr: ir.Expr, dtype: Optional[dt.Dtype], stype=None):
        self._expr = expr
        self._dtype = dtype
        self._stype = stype

    def _bin(self, op, other, swap=False):
        o = to_expr(other)
        e = ir.Bin(op, o, self._expr) if swap else ir.Bin(op, self._expr, o)
        return Value(e, _promote(self._dtype, other))

    def _cmp(self, op, other):
        return Value(ir.Bin(op, self._expr, to_expr(other)), dt.bool_)

    def __add__(self, o): return self._bin("+", o)
    def __radd__(self, o): return self._bin("+", o, True)
    def __sub__(self, o): return self._bin("-", o)
    def __rsub__(self, o): return self._bin("-", o, True)
    def __mul__(self, o): return self._bin("*", o)
    def __rmul__(self, o): return self._bin("*", o, True)
    def __truediv__(self, o): return self._bin("/", o)
    def __rtruediv__(self, o): return self._bin("/", o, True)
    def __floordiv__(self, o): return self._bin("/", o)
    def __rfloordiv__(self, o): return self._bin("/", o, True)
    def __mod__(self, o): return self._bin("%", o)
    def __rmod__(self, o): return self._bin("%", o, True)
    def __and__(self, o): return self._bin("&", o)
    def __rand__(self, o): return self._bin("&", o, True)
    def __or__(self, o): return self._bin("|", o)
    def __ror__(self, o): return self._bin("|", o, True)
    def __xor__(self, o): return self._bin("^", o)
    def __rxor__(self, o): return self._bin("^", o, True)
    def __lshift__(self, o): return self._bin("<<", o)
    def __rlshift__(self, o): return self._bin("<<", o, True)
    def __rshift__(self, o): return self._bin(">>", o)
    def __rrshift__(self, o): return self._bin(">>", o, True)

    def __lt__(self, o): return self._cmp("<", o)
    def __le__(self, o): return self._cmp("<=", o)
    def __gt__(self, o): return self._cmp(">", o)
    def __ge__(self, o): return self._cmp(">=", o)
    def __eq__(self, o): return self._cmp("==", o)
    def __ne__(self, o): return self._cmp("!=", o)

    def __neg__(self): return Value(ir.Unary("-", self._expr), self._dtype)
    def __pos__(self): return self
    def __invert__(self): return Value(ir.Unary("~", self._expr), self._dtype)

    def __bool__(self):
        raise TypeError(
            "Cannot use a traced thork value in a Python boolean context (e.g. `if`, `and`, "
            "`or`). Use kernel-level control flow (tk.if_, tk.while_) instead."
        )

    def __hash__(self):
        return id(self)


# reference names (tracer.py:207, 349) kept for code written against them
Tracer = Value


class Pointer:
    """A traced device pointer: ``p[i]`` loads, ``p[i] = v`` stores."""

    __slots__ = ("_expr", "_dtype", "_builder")

    def __init__(self, expr: ir.Expr, dtype: dt.Dtype, builder: KernelBuilder):
        self._expr = expr
        self._dtype = dtype
        self._builder = builder

    def __getitem__(self, index) -> Value:
        return Value(ir.Index(self._expr, to_expr(index)), self._dtype)

    def __setitem__(self, index, value) -> None:
        self._builder.add_stmt(ir.StoreStmt(ir.Index(self._expr, to_expr(index)), to_expr(value)))
        self._builder.mark_written(self._expr)


PointerTracer = Pointer


class Vector:
    """A traced uint2/uint3/int2/int3 value; ``.x/.y/.z/.w`` give scalars."""

    __slots__ = ("_expr", "_dtype", "_vec_size")
    _FIELDS = ("x", "y", "z", "w")

    def __init__(self, expr: ir.Expr, elem_dtype: dt.Dtype, vec_size: int):
        self._expr = expr
        self._dtype = elem_dtype
        self._vec_size = vec_size

    def __getattr__(self, name):
        if name in Vector._FIELDS:
            if Vector._FIELDS.index(name) >= self._vec_size:
                raise AttributeError(f"Vector of size {self._vec_size} has no field .{name}")
            return Value(ir.Field(self._expr, name), self._dtype)
        raise AttributeError(name)


VectorTracer = Vector


class Local(Value):
    """A mutable local from ``tk.local``; compound assignment emits updates."""

    __slots__ = ("_builder", "_name")

    def __init__(self, name: str, dtype: dt.Dtype, builder: KernelBuilder):
        super().__init__(ir.Name(name), dtype)
        self._builder = builder
        self._name = name

    def _update(self, op, value):
        self._builder.add_stmt(ir.AssignStmt(self._name, op, to_expr(value)))
        return self

    def __iadd__(self, o): return self._update("+=", o)
    def __isub__(self, o): return self._update("-=", o)
    def __imul__(self, o): return self._update("*=", o)
    def __itruediv__(self, o): return self._update("/=", o)
    def __ifloordiv__(self, o): return self._update("/=", o)
    def __imod__(self, o): return self._update("%=", o)
    def __iand__(self, o): return self._update("&=", o)
    def __ior__(self, o): return self._update("|=", o)
    def __ixor__(self, o): return self._update("^=", o)
    def __ilshift__(self, o): return self._update("<<=", o)
    def __irshift__(self, o): return self._update(">>=", o)

    def assign(self, value) -> None:
        """``name = value;``"""
        self._update("=", value)


def local(dtype: dt.Dtype, init) -> Local:
    """Declare ``T vN = init;`` and return a mutable handle."""
    b = current_builder()
    name = b.fresh_name("v")
    b.add_stmt(ir.Decl(name, dtype.cuda, init=to_expr(init)))
    return Local(name, dtype, b)


# --------------------------------------------------------------------------
# control flow
# --------------------------------------------------------------------------
class _Range:
    __slots__ = ("_start", "_stop", "_step")

    def __init__(self, start, stop, step):
        self._start, self._stop, self._step = start, stop, step

    def __iter__(self):
        b = current_builder()
        var = b.fresh_name("i")
        loc = user_location()
        b.open_block()
        try:
            yield Value(ir.Name(var), dt.uint32)
        finally:
            body = b.close_block()
            stmt = ir.For(var, self._start, self._stop, self._step, body)
            stmt.loc = loc
            b.add_stmt(stmt)


def range(*args):  # noqa: A001 - mirrors the reference's tk.range
    """``for i in tk.range([start,] end[, step])`` emits a C ``for`` loop.

    The body runs once at trace time; bounds may be ints or traced values.
    """
    if len(args) == 1:
        return _Range(ir.Lit(0), to_expr(args[0]), ir.Lit(1))
    if len(args) == 2:
        return _Range(to_expr(args[0]), to_expr(args[1]), ir.Lit(1))
    if len(args) == 3:
        return _Range(to_expr(args[0]), to_expr(args[1]), to_expr(args[2]))
    raise TypeError(f"tk.range expects 1-3 arguments, got {len(args)}")


class _IfBlock:
    def __init__(self, cond: ir.Expr):
        self._cond = cond
        self._stmt: Optional[ir.If] = None
        self._builder = None
        self._loc = None

    def __enter__(self):
        self._builder = current_builder()
        self._loc = user_location()
        self._builder.open_block()
        return self

    def __exit__(self, exc_type, exc, tb):
        body = self._builder.close_block()
        self._stmt = ir.If(self._cond, body, None)
        self._stmt.loc = self._loc
        self._builder.add_stmt(self._stmt)
        return False

    def else_(self) -> "_ElseBlock":
        """The matching ``else`` block; must directly follow the if-block."""
        if self._stmt is None:
            raise RuntimeError(
                "tk.if_(...).else_() can only be used after the if-block has been exited."
            )
        return _ElseBlock(self)


class _ElseBlock:
    def __init__(self, if_block: _IfBlock):
        self._if = if_block
        self._builder = None

    def __enter__(self):
        b = current_builder()
        if b.last_stmt() is not self._if._stmt:
            raise RuntimeError(
                "tk.else_ block must immediately follow its matching tk.if_ block "
                "(no statements in between)."
            )
        self._builder = b
        b.open_block()
        return self

    def __exit__(self, exc_type, exc, tb):
        self._if._stmt.orelse = self._builder.close_block()
        return False


def if_(cond) -> _IfBlock:
    """``with tk.if_(cond):`` emits ``if (cond) { ... }``; pair with
    ``.else_()`` for the else branch."""
    return _IfBlock(to_expr(cond))


class _WhileBlock:
    def __init__(self, cond: ir.Expr):
        self._cond = cond
        self._builder = None
        self._loc = None

    def __enter__(self):
        self._builder = current_builder()
        self._loc = user_location()
        self._builder.open_block()
        return self

    def __exit__(self, exc_type, exc, tb):
        stmt = ir.While(self._cond, self._builder.close_block())
        stmt.loc = self._loc
        self._builder.add_stmt(stmt)
        return False


def while_(cond) -> _WhileBlock:
    """``with tk.while_(cond):`` emits ``while (cond) { ... }``."""
    return _WhileBlock(to_expr(cond))


def break_() -> None:
    current_builder().add_stmt(ir.Jump("break"))


def continue_() -> None:
    current_builder().add_stmt(ir.Jump("continue"))


# --------------------------------------------------------------------------
# shared memory and barriers
# --------------------------------------------------------------------------
class SharedArray:
    """A statically sized ``__shared__`` array; ``a[i, j]`` == ``a[i][j]``."""

    __slots__ = ("_name", "_dtype", "_shape", "_builder", "_expr")

    def __init__(self, name, dtype, shape, builder):
        self._name, self._dtype, self._shape, self._builder = name, dtype, shape, builder
        self._expr = ir.Name(name)

    def _path(self, index) -> ir.Expr:
        idx = index if isinstance(index, tuple) else (index,)
        e = self._expr
        for i in idx:
            e = ir.Index(e, to_expr(i))
        return e

    def __getitem__(self, index) -> Value:
        return Value(self._path(index), self._dtype)

    def __setitem__(self, index, value) -> None:
        self._builder.add_stmt(ir.StoreStmt(self._path(index), to_expr(value)))


def shared(dtype: dt.Dtype, shape) -> SharedArray:
    """Declare ``__shared__ T sN[d0][d1]...`` (dims must be positive ints)."""
    b = current_builder()
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    for d in shape:
        if not isinstance(d, int) or isinstance(d, bool) or d <= 0:
            raise TypeError(f"shared array shape must be positive Python ints, got {shape!r}")
    name = b.fresh_name("s")
    b.add_stmt(ir.Decl(name, dtype.cuda, qual="__shared__", dims=shape))
    return SharedArray(name, dtype, shape, b)


def syncthreads() -> None:
    current_builder().add_stmt(ir.ExprStatement(ir.CallExpr("__syncthreads")))


def syncwarp(mask: int = 0xFFFFFFFF) -> None:
    current_builder().add_stmt(ir.ExprStatement(ir.CallExpr("__syncwarp", [ir.Lit(int(mask))])))


# --------------------------------------------------------------------------
# warp intrinsics (results are materialised into locals so a later use inside
# divergent control flow does not re-execute the collective there)
# --------------------------------------------------------------------------
def _materialise(func: str, args, dtype: dt.Dtype, prefix="warp") -> Value:
    b = current_builder()
    name = b.fresh_name(prefix)
    b.add_stmt(ir.Decl(name, dtype.cuda, init=ir.CallExpr(func, [to_expr(a) for a in args])))
    return Value(ir.Name(name), dtype)


def _dtype_of(x, default=dt.float32) -> dt.Dtype:
    return x._dtype if isinstance(x, Value) and x._dtype is not None else default


def shfl_sync(x, src_lane, width: int = 32, mask: int = 0xFFFFFFFF) -> Value:
    return _materialise("__shfl_sync", [int(mask), x, src_lane, int(width)], _dtype_of(x))


def shfl_up_sync(x, delta, width: int = 32, mask: int = 0xFFFFFFFF) -> Value:
    return _materialise("__shfl_up_sync", [int(mask), x, delta, int(width)], _dtype_of(x))


def shfl_down_sync(x, delta, width: int = 32, mask: int = 0xFFFFFFFF) -> Value:
    return _materialise("__shfl_down_sync", [int(mask), x, delta, int(width)], _dtype_of(x))


def shfl_xor_sync(x, lane_mask, width: int = 32, mask: int = 0xFFFFFFFF) -> Value:
    return _materialise("__shfl_xor_sync", [int(mask), x, lane_mask, int(width)], _dtype_of(x))


def ballot_sync(predicate, mask: int = 0xFFFFFFFF) -> Value:
    return _materialise("__ballot_sync", [int(mask), predicate], dt.uint32)


def all_sync(predicate, mask: int = 0xFFFFFFFF) -> Value:
    return _materialise("__all_sync", [int(mask), predicate], dt.int32)


def any_sync(predicate, mask: int = 0xFFFFFFFF) -> Value:
    return _materialise("__any_sync", [int(mask), predicate], dt.int32)


def warp_sum(x, mask: int = 0xFFFFFFFF) -> Value:
    """Butterfly reduction of ``x`` over the 32 lanes (every lane gets the sum)."""
    b = current_builder()
    dtype = _dtype_of(x)
    acc = b.fresh_name("warp")
    b.add_stmt(ir.Decl(acc, dtype.cuda, init=to_expr(x)))
    off = 16
    while off:
        b.add_stmt(ir.AssignStmt(acc, "+=", ir.CallExpr(
            "__shfl_xor_sync", [ir.Lit(int(mask)), ir.Name(acc), ir.Lit(off), ir.Lit(32)])))
        off //= 2
    return Value(ir.Name(acc), dtype)


# --------------------------------------------------------------------------
# math intrinsics and casts (pure expressions)
# --------------------------------------------------------------------------
def _math(func: str, *args, dtype: Optional[dt.Dtype] = None) -> Value:
    if dtype is None:
        dtype = args[0]._dtype if isinstance(args[0], Value) else None
    return Value(ir.CallExpr(func, [to_expr(a) for a in args]), dtype)


def exp(x): return _math("expf", x)
def exp2(x): return _math("exp2f", x)
def log(x): return _math("logf", x)
def log2(x): return _math("log2f", x)
def log10(x): return _math("log10f", x)
def sqrt(x): return _math("sqrtf", x)
def rsqrt(x): return _math("rsqrtf", x)
def sin(x): return _math("sinf", x)
def cos(x): return _math("cosf", x)
def tan(x): return _math("tanf", x)
def asin(x): return _math("asinf", x)
def acos(x): return _math("acosf", x)
def atan(x): return _math("atanf", x)
def sinh(x): return _math("sinhf", x)
def cosh(x): return _math("coshf", x)
def tanh(x): return _math("tanhf", x)
def floor(x): return _math("floorf", x)
def ceil(x): return _math("ceilf", x)
def round(x): return _math("roundf", x)  # noqa: A001
def trunc(x): return _math("truncf", x)
def fabs(x): return _math("fabsf", x)
def abs(x): return _math("abs", x)  # noqa: A001
def pow(x, y): return _math("powf", x, y)  # noqa: A001
def fmod(x, y): return _math("fmodf", x, y)
def atan2(y, x): return _math("atan2f", y, x)
def fmin(x, y): return _math("fminf", x, y)
def fmax(x, y): return _math("fmaxf", x, y)
def min(x, y): return _math("min", x, y)  # noqa: A001
def max(x, y): return _math("max", x, y)  # noqa: A001
def fma(a, b, c): return _math("fmaf", a, b, c)
def fast_exp(x): return _math("__expf", x)
def fast_log(x): return _math("__logf", x)
def fast_log2(x): return _math("__log2f", x)
def fast_log10(x): return _math("__log10f", x)
def fast_sqrt(x): return _math("__fsqrt_rn", x)
def fast_rsqrt(x): return _math("__frsqrt_rn", x)
def fast_sin(x): return _math("__sinf", x)
def fast_cos(x): return _math("__cosf", x)
def fast_tan(x): return _math("__tanf", x)
def fast_pow(x, y): return _math("__powf", x, y)


def cast(value, dtype: dt.Dtype) -> Value:
    """``static_cast<T>(value)``."""
    return Value(ir.CastTo(dtype.cuda, to_expr(value)), dtype)


# --------------------------------------------------------------------------
# atomics (the old value is always captured so the side effect is emitted)
# --------------------------------------------------------------------------
def _atomic(func: str, ptr, idx, *vals) -> Value:
    if not isinstance(ptr, Pointer):
        raise TypeError(f"atomic operations expect a tk.DevicePointer, got {type(ptr).__name__}")
    b = current_builder()
    addr = ir.AddressOf(ir.Index(ptr._expr, to_expr(idx)))
    name = b.fresh_name("atom")
    b.add_stmt(ir.Decl(name, ptr._dtype.cuda, init=ir.CallExpr(func, [addr] + [to_expr(v) for v in vals])))
    b.mark_written(ptr._expr)
    return Value(ir.Name(name), ptr._dtype)


def atomic_add(ptr, idx, value): return _atomic("atomicAdd", ptr, idx, value)
def atomic_sub(ptr, idx, value): return _atomic("atomicSub", ptr, idx, value)
def atomic_and(ptr, idx, value): return _atomic("atomicAnd", ptr, idx, value)
def atomic_or(ptr, idx, value): return _atomic("atomicOr", ptr, idx, value)
def atomic_xor(ptr, idx, value): return _atomic("atomicXor", ptr, idx, value)
def atomic_min(ptr, idx, value): return _atomic("atomicMin", ptr, idx, value)
def atomic_max(ptr, idx, value): return _atomic("atomicMax", ptr, idx, value)
def atomic_exch(ptr, idx, value): return _atomic("atomicExch", ptr, idx, value)


def atomic_cas(ptr, idx, compare, value) -> Value:
    """``atomicCAS(&ptr[idx], compare, value)``; returns the old value."""
    return _atomic("atomicCAS", ptr, idx, compare, value)


# --------------------------------------------------------------------------
# device functions
# --------------------------------------------------------------------------
class DeviceFn:
    """A ``__device__`` helper traced once, on its first call from a kernel.

    Parameters are annotated ``tk.DevicePointer[dtype]`` or a dtype; the
    return annotation (a dtype, or nothing for void) sets the return type.
    """

    def __init__(self, fn: Callable):
        self._fn = fn
        self._name = fn.__name__
        self._sig = inspect.signature(fn)
        self._traced = False
        self._tracing = False
        self._param_strs: List[str] = []
        self._return_type = "void"
        self._return_dtype: Optional[dt.Dtype] = None
        self._stmts: List[ir.Stmt] = []
        self._includes: List[tuple] = []
        self._deps: List["DeviceFn"] = []

    def _ensure_traced(self) -> None:
        if self._traced:
            return
        if self._tracing:
            raise RuntimeError(
                f"Device fn '{self._name}' is recursive; CUDA does not support recursion in "
                "__device__ functions"
            )
        self._tracing = True
        try:
            self._trace()
            self._traced = True
        finally:
            self._tracing = False

    def _trace(self) -> None:
        b = KernelBuilder(self._name)
        args, strs = [], []
        for pname, p in self._sig.parameters.items():
            if p.kind in (inspect.Parameter.VAR_POSITIONAL, inspect.Parameter.VAR_KEYWORD):
                raise TypeError(f"Device fn '{self._name}': *args/**kwargs not supported")
            ann = p.annotation
            if ann is inspect.Parameter.empty:
                raise TypeError(
                    f"Device fn '{self._name}': parameter '{pname}' is missing a type annotation")
            if isinstance(ann, DevicePointerSpec):
                strs.append(f"{ann.dtype.cuda} *{pname}")
                args.append(Pointer(ir.Name(pname), ann.dtype, b))
            elif isinstance(ann, dt.Dtype):
                strs.append(f"{ann.cuda} {pname}")
                args.append(Value(ir.Name(pname), ann))
            else:
                raise TypeError(
                    f"Device fn '{self._name}': parameter '{pname}' has unsupported annotation "
                    f"{ann!r}. Expected tk.DevicePointer[...] or a thork dtype.")
        ret = self._sig.return_annotation
        if ret in (inspect.Parameter.empty, None, type(None)):
            rtype, rdtype = "void", None
        elif isinstance(ret, dt.Dtype):
            rtype, rdtype = ret.cuda, ret
        else:
            raise TypeError(
                f"Device fn '{self._name}': return annotation must be a thork dtype or omitted, "
                f"got {ret!r}")
        token = _active.set(b)
        try:
            result = self._fn(*args)
        finally:
            _active.reset(token)
        if rdtype is not None:
            if result is None:
                raise TypeError(
                    f"Device fn '{self._name}' declared return type {rdtype.name} but returned None")
            b.add_stmt(ir.Jump("return", to_expr(result)))
        self._param_strs = strs
        self._return_type, self._return_dtype = rtype, rdtype
        self._stmts = b.stmts
        self._includes = list(b.includes)
        self._deps = list(b.device_functions)

    def __call__(self, *args):
        b = current_builder()
        b.add_device_fn(self)
        if len(args) != len(self._param_strs):
            raise TypeError(
                f"Device fn '{self._name}' expected {len(self._param_strs)} argument(s), "
                f"got {len(args)}")
        call = ir.CallExpr(self._name, [to_expr(a) for a in args])
        if self._return_dtype is None:
            b.add_stmt(ir.ExprStatement(call))
            return None
        return Value(call, self._return_dtype)


def device_fn(fn: Callable) -> DeviceFn:
    """Decorator: make ``fn`` a reusable ``__device__`` function."""
    return DeviceFn(fn)


# the builtin range stays reachable for code in this module
_py_range = builtins.range
