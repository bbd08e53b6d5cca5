"""Kernel IR: the expression/statement tree that tracing builds and
``codegen`` prints as CUDA C++.

Plays the role of the reference's ``src/thork/ir.py`` (expressions ``ir.py:8-98``,
statements ``ir.py:101-230``, parameters ``ir.py:233-242``) with a smaller
node set: declarations of every flavour are one ``Decl`` node and all jumps
one ``Jump`` node.  Every statement carries ``loc`` = (python file, line) of
the user code that produced it, which feeds the generated-line source map.
"""

from dataclasses import dataclass, field
from typing import List, Optional, Tuple, Type, Union

from . import dtypes as dt
from .types import ThreadAttribute


# ---------------------------------------------------------------- expressions
class Expr:
    __slots__ = ()


@dataclass
class Name(Expr):
    name: str


@dataclass
class Lit(Expr):
    value: Union[int, float, bool]


@dataclass
class Index(Expr):
    """``base[index]``."""

    base: Expr
    index: Expr


@dataclass
class Field(Expr):
    """``base.field``."""

    base: Expr
    field: str


@dataclass
class Bin(Expr):
    op: str
    lhs: Expr
    rhs: Expr


@dataclass
class Unary(Expr):
    op: str
    operand: Expr


@dataclass
class AddressOf(Expr):
    operand: Expr


@dataclass
class CastTo(Expr):
    ctype: str
    operand: Expr


@dataclass
class CallExpr(Expr):
    """``func<targs>(args)``; ``func`` may be a dotted/scoped C++ name."""

    func: str
    args: List[Expr] = field(default_factory=list)
    targs: List[str] = field(default_factory=list)


@dataclass
class Verbatim(Expr):
    """CUDA text embedded as-is."""

    text: str


# ---------------------------------------------------------------- statements
class Stmt:
    loc: Optional[Tuple[str, int]] = None


@dataclass
class StoreStmt(Stmt):
    """``target = value;`` where target is an Index/Field/Name lvalue."""

    target: Expr
    value: Expr


@dataclass
class Decl(Stmt):
    """Declaration ``[qual] ctype name[dims] [= init | (ctor_args)];``."""

    name: str
    ctype: str
    init: Optional[Expr] = None
    qual: str = ""                 # e.g. "__shared__"
    dims: Tuple[int, ...] = ()
    ctor_args: Optional[List[Expr]] = None


@dataclass
class AssignStmt(Stmt):
    """``name op value;`` with op one of = += -= ..."""

    name: str
    op: str
    value: Expr


@dataclass
class ExprStatement(Stmt):
    expr: Expr


@dataclass
class For(Stmt):
    """``for (unsigned int var = start; var < stop; var += step) { body }``."""

    var: str
    start: Expr
    stop: Expr
    step: Expr
    body: List[Stmt] = field(default_factory=list)


@dataclass
class If(Stmt):
    cond: Expr
    then: List[Stmt] = field(default_factory=list)
    orelse: Optional[List[Stmt]] = None


@dataclass
class While(Stmt):
    cond: Expr
    body: List[Stmt] = field(default_factory=list)


@dataclass
class Jump(Stmt):
    """``break;`` / ``continue;`` / ``return [value];``."""

    kind: str
    value: Optional[Expr] = None


# ---------------------------------------------------------------- parameters
@dataclass
class Param:
    """A kernel parameter.

    kind: ``pointer`` (device buffer), ``constant`` (by-value scalar),
    ``attribute`` (built-in synthesised at entry, not passed) or
    ``kittens_global`` (2-D tile-addressed global).  ``written`` marks
    buffers the kernel stores to; only those are copied back to the host
    (reference ``tracer.py:311-319``, ``runtime.py:693-696``).
    """

    name: str
    kind: str
    dtype: dt.Dtype
    cuda_name: Optional[str] = None
    vec_size: int = 1
    attribute: Optional[Type[ThreadAttribute]] = None
    written: bool = False
    tile_shape: Optional[Tuple[int, int]] = None

    @property
    def bindable(self) -> bool:
        return self.kind in ("pointer", "constant", "kittens_global")
