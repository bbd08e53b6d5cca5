"""IR -> CUDA C++ source, with a generated-line -> Python-line source map.

Counterpart of the reference's ``src/thork/codegen.py``: expression printing
with C precedence (``codegen.py:12-83``), statements (``101-209``), device
functions (``212-228``), kernel parameters and attribute locals
(``282-319``) and ``emit_kernel`` (``322-406``).  Tile-addressed globals
lower to this package's own device library (``thork_tk.cuh``) instead of
ThunderKittens types, and there is no generated host launcher
(``codegen.py:416-469``): every kernel launches through the runtime's
``thork_launch``.
"""

import math
from typing import Dict, List, Tuple

from . import ir

SourceMap = Dict[int, Tuple[str, int]]

_PREC = {
    "||": 4, "&&": 5, "|": 6, "^": 7, "&": 8,
    "==": 9, "!=": 9, "<": 10, "<=": 10, ">": 10, ">=": 10,
    "<<": 11, ">>": 11, "+": 12, "-": 12, "*": 13, "/": 13, "%": 13,
}
_UNARY_PREC = 15
_POSTFIX_PREC = 16


def format_literal(v) -> str:
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, int):
        if v < 0:
            return f"({v})" if v >= -(2 ** 31) else f"({v}ll)"
        if v <= 2 ** 31 - 1:
            return str(v)
        if v <= 2 ** 32 - 1:
            return f"{v}u"
        return f"{v}ull"
    if isinstance(v, float):
        if math.isnan(v):
            return "__int_as_float(0x7fffffff)"
        if math.isinf(v):
            return "__int_as_float(0x7f800000)" if v > 0 else "__int_as_float(0xff800000)"
        text = repr(v)
        if "e" not in text and "." not in text:
            text += ".0"
        return text + "f"
    raise TypeError(f"Cannot format constant of type {type(v).__name__}: {v!r}")


def _prec(e: ir.Expr) -> int:
    if isinstance(e, ir.Bin):
        return _PREC.get(e.op, 0)
    if isinstance(e, (ir.Unary, ir.AddressOf, ir.CastTo)):
        return _UNARY_PREC
    if isinstance(e, ir.Lit) and isinstance(e.value, (int, float)) and not isinstance(e.value, bool):
        return _POSTFIX_PREC
    if isinstance(e, ir.Verbatim):
        return 0
    return _POSTFIX_PREC


def format_expr(e: ir.Expr, parent: int = 0, right: bool = False) -> str:
    """Render an expression; parenthesise when the parent binds tighter."""
    if isinstance(e, ir.Name):
        s = e.name
    elif isinstance(e, ir.Lit):
        s = format_literal(e.value)
    elif isinstance(e, ir.Index):
        s = f"{format_expr(e.base, _POSTFIX_PREC)}[{format_expr(e.index)}]"
    elif isinstance(e, ir.Field):
        s = f"{format_expr(e.base, _POSTFIX_PREC)}.{e.field}"
    elif isinstance(e, ir.Bin):
        p = _PREC.get(e.op)
        if p is None:
            raise TypeError(f"Unknown binary operator {e.op!r}")
        s = f"{format_expr(e.lhs, p)} {e.op} {format_expr(e.rhs, p, right=True)}"
    elif isinstance(e, ir.Unary):
        s = f"{e.op}{format_expr(e.operand, _UNARY_PREC)}"
    elif isinstance(e, ir.AddressOf):
        s = f"&{format_expr(e.operand, _UNARY_PREC)}"
    elif isinstance(e, ir.CastTo):
        s = f"static_cast<{e.ctype}>({format_expr(e.operand)})"
    elif isinstance(e, ir.CallExpr):
        t = f"<{', '.join(str(a) for a in e.targs)}>" if e.targs else ""
        s = f"{e.func}{t}({', '.join(format_expr(a) for a in e.args)})"
    elif isinstance(e, ir.Verbatim):
        return e.text
    else:
        raise TypeError(f"Unknown expression node: {type(e).__name__}")
    p = _prec(e)
    if p < parent or (right and p == parent and p < _UNARY_PREC):
        s = f"({s})"
    return s


class _Emitter:
    """Collects output lines and the source location of each."""

    def __init__(self):
        self.lines: List[str] = []
        self.smap: SourceMap = {}

    def put(self, text: str, loc=None) -> None:
        self.lines.append(text)
        if loc:
            self.smap[len(self.lines)] = loc

    def stmts(self, stmts: List[ir.Stmt], depth: int) -> None:
        for s in stmts:
            self.stmt(s, depth)

    def block(self, body: List[ir.Stmt], depth: int) -> None:
        pad = "    " * depth
        self.put(pad + "{")
        if body:
            self.stmts(body, depth + 1)
        else:
            self.put(pad + "    // empty")
        self.put(pad + "}")

    def stmt(self, s: ir.Stmt, depth: int) -> None:
        pad = "    " * depth
        loc = getattr(s, "loc", None)
        if isinstance(s, ir.StoreStmt):
            self.put(f"{pad}{format_expr(s.target)} = {format_expr(s.value)};", loc)
        elif isinstance(s, ir.Decl):
            q = f"{s.qual} " if s.qual else ""
            dims = "".join(f"[{d}]" for d in s.dims)
            if s.ctor_args is not None:
                args = ", ".join(format_expr(a) for a in s.ctor_args)
                tail = f"({args})" if s.ctor_args else "{}"
                self.put(f"{pad}{q}{s.ctype} {s.name}{dims}{tail};", loc)
            elif s.init is not None:
                self.put(f"{pad}{q}{s.ctype} {s.name}{dims} = {format_expr(s.init)};", loc)
            else:
                self.put(f"{pad}{q}{s.ctype} {s.name}{dims};", loc)
        elif isinstance(s, ir.AssignStmt):
            self.put(f"{pad}{s.name} {s.op} {format_expr(s.value)};", loc)
        elif isinstance(s, ir.ExprStatement):
            self.put(f"{pad}{format_expr(s.expr)};", loc)
        elif isinstance(s, ir.Jump):
            if s.value is not None:
                self.put(f"{pad}{s.kind} {format_expr(s.value)};", loc)
            else:
                self.put(f"{pad}{s.kind};", loc)
        elif isinstance(s, ir.For):
            step = (f"{s.var}++" if isinstance(s.step, ir.Lit) and s.step.value == 1
                    else f"{s.var} += {format_expr(s.step)}")
            self.put(f"{pad}for (unsigned int {s.var} = {format_expr(s.start)}; "
                     f"{s.var} < {format_expr(s.stop)}; {step})", loc)
            self.block(s.body, depth)
        elif isinstance(s, ir.While):
            self.put(f"{pad}while ({format_expr(s.cond)})", loc)
            self.block(s.body, depth)
        elif isinstance(s, ir.If):
            self.put(f"{pad}if ({format_expr(s.cond)})", loc)
            self.block(s.then, depth)
            if s.orelse is not None:
                self.put(f"{pad}else")
                self.block(s.orelse, depth)
        else:
            raise TypeError(f"Unknown statement node: {type(s).__name__}")


def format_stmts(stmts: List[ir.Stmt], indent: int = 4) -> Tuple[str, Dict[int, tuple]]:
    """CUDA text of ``stmts`` indented by ``indent`` spaces, and a map from
    0-indexed line within the text to the Python source location
    (reference ``codegen.py:191-202``)."""
    em = _Emitter()
    em.stmts(list(stmts), 0)
    pad = " " * indent
    text = "\n".join(pad + line for line in em.lines)
    return text, {line - 1: loc for line, loc in em.smap.items()}


def format_stmt(stmt: ir.Stmt, indent: int = 4) -> Tuple[str, Dict[int, tuple]]:
    """``format_stmts`` of a single statement (reference ``codegen.py:101``)."""
    return format_stmts([stmt], indent)


def _param_decl(p: ir.Param) -> str:
    if p.kind == "pointer":
        return f"{p.dtype.cuda} *{p.name}"
    if p.kind == "constant":
        return f"{p.cuda_name or p.dtype.cuda} {p.name}"
    if p.kind == "kittens_global":
        return f"const __grid_constant__ {global_type(p)} {p.name}"
    raise ValueError(f"Param kind {p.kind!r} is not a kernel argument")


def global_type(p: ir.Param) -> str:
    """Device-library type of a tile-addressed global parameter."""
    from .kittens import elem_ctype  # local import: kittens imports codegen helpers
    r, c = p.tile_shape if p.tile_shape else (0, 0)
    return f"thork::tk::gl<{elem_ctype(p.dtype)}, {r}, {c}>"


def _attribute_init(p: ir.Param) -> str:
    attr = p.attribute
    base = attr.cuda_expr
    if not attr.vector:
        return base
    if p.vec_size == 1:
        return f"{base}.x"
    comps = ("x", "y", "z")[: p.vec_size]
    signed = p.dtype.is_signed
    vals = ", ".join(f"static_cast<int>({base}.{c})" if signed else f"{base}.{c}" for c in comps)
    return f"make_{p.cuda_name}({vals})"


STATUS_PARAM = "__thork_status"


def emit_device_fn(df, em: _Emitter) -> None:
    em.put(f"static __device__ {df._return_type} {df._name}({', '.join(df._param_strs)})")
    em.block(df._stmts, 0)


def emit_kernel(builder) -> Tuple[str, SourceMap]:
    """Render the full CUDA source of a traced kernel.

    Returns (source, source_map) where source_map maps 1-based generated
    line numbers to (python file, line) of the statement that produced them.
    """
    em = _Emitter()
    for path, system in builder.includes:
        em.put(f"#include <{path}>" if system else f'#include "{path}"')
    em.put("")
    for df in builder.device_functions:
        emit_device_fn(df, em)
        em.put("")

    decls = [_param_decl(p) for p in builder.params if p.bindable]
    if builder.uses_status:
        decls.append(f"unsigned int *{STATUS_PARAM}")
    em.put(f'extern "C" __global__ void {builder.name}(')
    if decls:
        for d in decls[:-1]:
            em.put(f"    {d},")
        em.put(f"    {decls[-1]})")
    else:
        em.put(")")
    em.put("{")
    attrs = [p for p in builder.params if p.kind == "attribute"]
    for p in attrs:
        ctype = p.cuda_name if p.vec_size > 1 else p.dtype.cuda
        em.put(f"    const {ctype} {p.name} = {_attribute_init(p)};")
    for text in builder.prologue:
        em.put("    " + text)
    if builder.stmts:
        em.stmts(builder.stmts, 1)
    elif not attrs:
        em.put("    // empty kernel")
    for text in builder.epilogue:
        em.put("    " + text)
    em.put("}")
    return "\n".join(em.lines) + "\n", em.smap
