"""thork_b200.kittens — tile operations in the ThunderKittens vocabulary,
lowered to this package's own sm_100a tile library (``thork_tk.cuh``).

Front end of the reference's ``src/thork/kittens.py``: same names, argument
conventions, type checks and ``written`` marking (``kittens.py:105-857``).
What is emitted differs: instead of ``kittens::`` templates compiled by nvcc,
the calls target ``thork::tk::`` functions written for B200 (TMA tensor
maps, mbarriers with bounded waits, tcgen05 MMA into TMEM, mma.sync for
register tiles) and compile through NVRTC for sm_100a.

Storage decisions made at trace time:
* shared tiles (``st_*``) get fixed, 1024-byte-aligned offsets in the
  kernel's dynamic shared memory, whose size is computed exactly (the
  reference always requests the device maximum, ``jit.py:213``);
* TMEM tiles (``tt_*``) and semaphores are ``__shared__`` objects, so a value
  assigned by one thread (``tensor_alloc`` under a lane test) is seen by the
  whole block after a barrier;
* ``tensor_allocator`` allocates TMEM at its declaration and the kernel
  releases it before returning.
"""

from typing import Optional

from . import dtypes as dt
from . import ir
from .tracer import KernelBuilder, Value, current_builder, to_expr
from .types import KittensGlobal as Global  # noqa: F401  (re-export)

__all__ = [
    "Global", "KittensGlobalTracer", "RegisterTile", "SharedTile", "rt_bf", "rt_hf", "rt_fl",
    "rt_bf_col", "rt_hf_col", "rt_fl_col", "st_bf", "st_hf", "st_fl", "zero", "load", "store",
    "swap_layout", "mma_AB", "mma_AB_t", "warpgroup", "Semaphore", "semaphore",
    "init_semaphore", "wait", "tma", "TensorTile", "TensorAllocator", "tt_bf", "tt_hf",
    "tt_fl", "tensor_allocator", "tensor_alloc", "tcgen05_commit", "tensor_load_wait",
    "cluster_ctarank", "cluster_sync", "arrive",
]

_ELEM = {"float32": "float", "float16": "__half", "bfloat16": "__nv_bfloat16",
         "float8_e4m3": "unsigned char", "int32": "int", "uint32": "unsigned int"}
NS = "thork::tk"
SMEM_BASE = "__thork_smem"


def elem_ctype(d: dt.Dtype) -> str:
    if d.name not in _ELEM:
        raise TypeError(f"thork dtype {d.name} has no tile-library equivalent")
    return _ELEM[d.name]


# ---------------------------------------------------------------- hooks
_tk_stype_hooks = {}


def register_tk_stype_hooks(**hooks) -> None:
    """Registration point for a verification layer (reference
    ``kittens.py:82-92``); hooks are called after the matching op."""
    _tk_stype_hooks.update(hooks)


def _hook(name, *args):
    fn = _tk_stype_hooks.get(name)
    if fn is not None:
        fn(*args)


# ---------------------------------------------------------------- builder state
def mark_kittens(b: KernelBuilder) -> None:
    """Flag a kernel as a tile kernel: include the tile library and emit the
    per-CTA set-up / teardown."""
    if not b.uses_kittens:
        b.uses_kittens = True
        b.add_include("thork_tk.cuh", system=False)
        b.tk_smem_bytes = 0
        b.tk_min_smem = 0
        b.tk_epilogue = []
        b.tk_cluster = 1


def _mark_pair(b: KernelBuilder) -> None:
    """The kernel uses 2-CTA (cluster pair) operations: it must be launched
    with a cluster of (2, 1, 1)."""
    mark_kittens(b)
    b.tk_cluster = 2


def _mark_tma(b: KernelBuilder) -> None:
    mark_kittens(b)
    b.uses_tma = True


def finalize(b: KernelBuilder) -> None:
    """Complete a traced tile kernel: shared-memory base, bounded-wait
    status, set-up and teardown code, dynamic shared memory size."""
    pro = [f"{NS}::kernel_begin();"]
    if b.tk_smem_bytes:
        pro.insert(0, "extern __shared__ __align__(1024) unsigned char __thork_dsmem[];")
        pro.insert(1, f"unsigned char *{SMEM_BASE} = __thork_dsmem + "
                      "((1024u - (thork::dev::smem_u32(__thork_dsmem) & 1023u)) & 1023u);")
    b.prologue = pro + b.prologue
    b.epilogue = list(b.tk_epilogue) + [f"{NS}::kernel_end();"]
    b.dynamic_smem = max(b.tk_smem_bytes + (1024 if b.tk_smem_bytes else 0), b.tk_min_smem)
    if b.dynamic_smem and not b.tk_smem_bytes:
        b.prologue.insert(0, "extern __shared__ __align__(1024) unsigned char __thork_dsmem[];")


def _stmt(b: KernelBuilder, func: str, args, targs=None) -> None:
    b.add_stmt(ir.ExprStatement(ir.CallExpr(func, list(args), list(targs or []))))


# ---------------------------------------------------------------- handles
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


class RegisterTile(_Handle):
    __slots__ = ("_rows", "_cols", "_layout")

    def __init__(self, expr, dtype, builder, rows, cols, layout):
        super().__init__(expr, dtype, builder)
        self._rows, self._cols, self._layout = rows, cols, layout


class SharedTile(_Handle):
    __slots__ = ("_rows", "_cols")

    def __init__(self, expr, dtype, builder, rows, cols):
        super().__init__(expr, dtype, builder)
        self._rows, self._cols = rows, cols


class TensorTile(_Handle):
    __slots__ = ("_rows", "_cols", "_ncta")

    def __init__(self, expr, dtype, builder, rows, cols):
        super().__init__(expr, dtype, builder)
        self._rows, self._cols = rows, cols
        self._ncta = 1  # 2 once bound to a cluster-pair allocator


class TensorAllocator(_Handle):
    __slots__ = ("_ncta",)

    def __init__(self, name: str, builder: KernelBuilder, ncta: int = 1):
        super().__init__(ir.Name(name), dt.uint32, builder)
        self._ncta = ncta


class Semaphore(_Handle):
    __slots__ = ()

    def __init__(self, name: str, builder: KernelBuilder):
        super().__init__(ir.Name(name), dt.uint32, builder)


def _check_dims(alias: str, rows, cols) -> None:
    for v, label in ((rows, "rows"), (cols, "cols")):
        if not isinstance(v, int) or isinstance(v, bool) or v <= 0:
            raise TypeError(f"{alias} {label} must be a positive int, got {v!r}")


# ---------------------------------------------------------------- declarations
def _rt_factory(layout: int, alias: str, d: dt.Dtype):
    def make(rows: int, cols: int) -> RegisterTile:
        _check_dims(alias, rows, cols)
        if rows % 16 or cols % 16:
            raise TypeError(f"{alias} dims must be multiples of 16, got ({rows}, {cols})")
        b = current_builder()
        mark_kittens(b)
        name = b.fresh_name("rt")
        b.add_stmt(ir.Decl(name, f"{NS}::rt<{elem_ctype(d)}, {rows}, {cols}, {layout}>"))
        return RegisterTile(ir.Name(name), d, b, rows, cols, "row" if layout == 0 else "col")
    make.__name__ = alias
    return make


rt_bf = _rt_factory(0, "rt_bf", dt.bfloat16)
rt_hf = _rt_factory(0, "rt_hf", dt.float16)
rt_fl = _rt_factory(0, "rt_fl", dt.float32)
rt_bf_col = _rt_factory(1, "rt_bf_col", dt.bfloat16)
rt_hf_col = _rt_factory(1, "rt_hf_col", dt.float16)
rt_fl_col = _rt_factory(1, "rt_fl_col", dt.float32)


def _st_factory(alias: str, d: dt.Dtype):
    def make(rows: int, cols: int) -> SharedTile:
        _check_dims(alias, rows, cols)
        if rows % 8 or (cols * d.nbytes) % 16:
            raise TypeError(
                f"{alias} needs rows % 8 == 0 and 16-byte rows, got ({rows}, {cols})")
        b = current_builder()
        mark_kittens(b)
        name = b.fresh_name("st")
        off = b.tk_smem_bytes
        b.tk_smem_bytes = off + ((rows * cols * d.nbytes + 1023) // 1024) * 1024
        ctype = f"{NS}::st<{elem_ctype(d)}, {rows}, {cols}>"
        b.add_stmt(ir.Decl(name, f"{ctype} &",
                           init=ir.Verbatim(f"*reinterpret_cast<{ctype} *>({SMEM_BASE} + {off})")))
        return SharedTile(ir.Name(name), d, b, rows, cols)
    make.__name__ = alias
    return make


st_bf = _st_factory("st_bf", dt.bfloat16)
st_hf = _st_factory("st_hf", dt.float16)
st_fl = _st_factory("st_fl", dt.float32)


def _tt_factory(alias: str, d: dt.Dtype):
    def make(rows: int, cols: int) -> TensorTile:
        _check_dims(alias, rows, cols)
        b = current_builder()
        mark_kittens(b)
        name = b.fresh_name("tt")
        b.add_stmt(ir.Decl(name, f"{NS}::tt<{elem_ctype(d)}, {rows}, {cols}>", qual="__shared__"))
        return TensorTile(ir.Name(name), d, b, rows, cols)
    make.__name__ = alias
    return make


tt_bf = _tt_factory("tt_bf", dt.bfloat16)
tt_hf = _tt_factory("tt_hf", dt.float16)
tt_fl = _tt_factory("tt_fl", dt.float32)


def tensor_allocator(nblocks_per_sm: int = 1, ncta: int = 1) -> TensorAllocator:
    """Allocate this CTA's share of tensor memory (512 / nblocks_per_sm
    columns); it is released when the kernel finishes.  Must be reached by
    every thread of the block (top level of the kernel).

    ``ncta=2`` allocates for a CTA pair (``tcgen05.alloc.cta_group::2`` in
    both CTAs): the kernel must then be launched with a cluster of
    ``(2, 1, 1)`` (``kernel[grid, block, (2, 1, 1)]``), tiles bound to this
    allocator take the 2-CTA MMA forms, and the allocation also serves as the
    cluster barrier that makes both CTAs' semaphores visible to each other
    (initialise them before it)."""
    if nblocks_per_sm not in (1, 2) or ncta not in (1, 2):
        raise ValueError("tensor_allocator: nblocks_per_sm and ncta must each be 1 or 2")
    b = current_builder()
    mark_kittens(b)
    name = b.fresh_name("tm")
    cols = 512 // nblocks_per_sm
    # Each CTA takes 512/nblocks_per_sm TMEM columns; reserving more than
    # 1/(nblocks_per_sm+1) of the SM's 228 KiB of shared memory keeps any
    # further CTA off the SM, so allocations never contend.
    b.tk_min_smem = max(b.tk_min_smem, (120 if nblocks_per_sm == 1 else 80) * 1024)
    b.add_stmt(ir.Decl(name, "unsigned int", qual="__shared__"))
    if ncta == 2:
        _mark_pair(b)
        _stmt(b, f"{NS}::tmem_acquire2<{cols}>", [ir.Verbatim(f"&{name}")])
        b.tk_epilogue.append(f"{NS}::tmem_release2<{cols}>(&{name});")
    else:
        _stmt(b, f"{NS}::tmem_acquire<{cols}>", [ir.Verbatim(f"&{name}")])
        b.tk_epilogue.append(f"{NS}::tmem_release<{cols}>(&{name});")
    return TensorAllocator(name, b, ncta)


def tensor_alloc(tt: TensorTile, alloc: TensorAllocator, col_offset=0) -> None:
    """Bind ``tt`` to columns of ``alloc`` starting at ``col_offset`` (one
    thread may do it; others see it after a barrier)."""
    if not isinstance(tt, TensorTile):
        raise TypeError("tensor_alloc tt must be a TensorTile")
    if not isinstance(alloc, TensorAllocator):
        raise TypeError("tensor_alloc alloc must be a TensorAllocator")
    b = current_builder()
    mark_kittens(b)
    tt._ncta = alloc._ncta
    b.add_stmt(ir.AssignStmt(tt._expr.name, "=", ir.CallExpr(
        f"{NS}::tensor_alloc", [alloc._expr, to_expr(col_offset)],
        [f"decltype({tt._expr.name})"])))


def tcgen05_commit(sem: Semaphore, ncta: int = 1) -> None:
    """Arrive on ``sem`` once every tcgen05 op issued so far by this thread
    has completed (issue from the thread that issued the MMAs).  With
    ``ncta=2`` (the pair leader's MMA thread) the arrival lands on ``sem`` in
    both CTAs of the pair."""
    if not isinstance(sem, Semaphore):
        raise TypeError("tcgen05_commit sem must be a Semaphore")
    if ncta not in (1, 2):
        raise ValueError("tcgen05_commit ncta must be 1 or 2")
    b = current_builder()
    if ncta == 2:
        _mark_pair(b)
    else:
        mark_kittens(b)
    _stmt(b, f"{NS}::tcgen05_commit<{ncta}>", [sem._expr])


def cluster_ctarank() -> Value:
    """This CTA's rank in its cluster (0 or 1 for a pair; 0 without a
    cluster launch)."""
    b = current_builder()
    mark_kittens(b)
    name = b.fresh_name("ctarank")
    b.add_stmt(ir.Decl(name, "int", init=ir.CallExpr(f"{NS}::cluster_ctarank")))
    return Value(ir.Name(name), dt.int32)


def cluster_sync() -> None:
    """Barrier over every thread of every CTA in the cluster."""
    b = current_builder()
    mark_kittens(b)
    _stmt(b, f"{NS}::cluster_sync", [])


def tensor_load_wait() -> None:
    """Wait for outstanding tensor-memory loads of this thread."""
    b = current_builder()
    mark_kittens(b)
    _stmt(b, f"{NS}::tensor_load_wait", [])


def semaphore() -> Semaphore:
    """Declare a shared mbarrier; initialise it with ``init_semaphore`` from
    one thread, then synchronise the block."""
    b = current_builder()
    mark_kittens(b)
    name = b.fresh_name("sem")
    b.add_stmt(ir.Decl(name, f"{NS}::semaphore", qual="__shared__"))
    return Semaphore(name, b)


def init_semaphore(sem: Semaphore, n_arrived: int, n_threads: int) -> None:
    """Initialise ``sem`` to complete a phase after ``n_arrived + n_threads``
    arrivals (transaction bytes counted separately via ``tma.expect_bytes``)."""
    if not isinstance(sem, Semaphore):
        raise TypeError("init_semaphore expects a kittens.semaphore handle")
    b = current_builder()
    mark_kittens(b)
    _stmt(b, f"{NS}::init_semaphore", [sem._expr, ir.Lit(int(n_arrived)), ir.Lit(int(n_threads))])


def arrive(sem: Semaphore) -> None:
    """Arrive once on ``sem`` from the calling thread (ThunderKittens'
    ``kittens::arrive``; no counterpart in the reference's front end).  Earlier
    tensor-memory reads of the thread are ordered before the arrival, so it
    can hand an accumulator back to the MMA issuer."""
    if not isinstance(sem, Semaphore):
        raise TypeError("arrive expects a kittens.semaphore handle")
    b = current_builder()
    mark_kittens(b)
    _stmt(b, f"{NS}::arrive", [sem._expr])


def wait(sem: Semaphore, phase) -> None:
    """Block until the phase of ``sem`` with parity ``phase`` completes.  The
    wait is bounded: on expiry it records a status the launch reports."""
    if not isinstance(sem, Semaphore):
        raise TypeError("wait expects a kittens.semaphore handle")
    b = current_builder()
    mark_kittens(b)
    b.uses_status = True
    _stmt(b, f"{NS}::wait", [sem._expr, to_expr(phase), ir.Verbatim("__thork_status")])


def _coord(coord) -> ir.Expr:
    if not (isinstance(coord, tuple) and len(coord) == 2):
        raise TypeError(f"kittens load/store coord must be a (row, col) tuple, got {coord!r}")
    from .codegen import format_expr
    r, c = coord
    return ir.Verbatim(f"{NS}::coord{{static_cast<int>({format_expr(to_expr(r))}), "
                       f"static_cast<int>({format_expr(to_expr(c))})}}")


# ---------------------------------------------------------------- warp / warpgroup ops
def _zero(scope: str, rt) -> None:
    if not isinstance(rt, RegisterTile):
        raise TypeError(f"kittens.zero expects a register tile, got {type(rt).__name__}")
    b = current_builder()
    mark_kittens(b)
    _stmt(b, f"{NS}::{scope}::zero", [rt._expr])
    _hook("zero", rt)


def _load(scope: str, dst, src, coord) -> None:
    b = current_builder()
    mark_kittens(b)
    if isinstance(dst, SharedTile) and isinstance(src, GlobalHandle):
        if coord is None:
            raise TypeError("load(shared, global, coord) requires a coord tuple")
        _check_elem(dst, src)
        _stmt(b, f"{NS}::{scope}::load", [dst._expr, src._expr, _coord(coord)])
    elif isinstance(dst, RegisterTile) and isinstance(src, SharedTile):
        if coord is not None:
            raise TypeError("load(register, shared) does not take a coord")
        if dst._dtype.nbytes != 2 or src._dtype != dst._dtype:
            raise TypeError("load(register, shared) moves 16-bit tiles of the same type")
        _stmt(b, f"{NS}::{scope}::load", [dst._expr, src._expr])
    elif isinstance(dst, RegisterTile) and isinstance(src, GlobalHandle):
        if coord is None:
            raise TypeError("load(register, global, coord) requires a coord tuple")
        if scope != "warp" or dst._layout != "row":
            raise TypeError("load(register, global) is warp-scoped into a row-layout tile")
        _stmt(b, f"{NS}::{scope}::load", [dst._expr, src._expr, _coord(coord)])
    else:
        raise TypeError(
            f"kittens.load: unsupported argument combination "
            f"({type(dst).__name__}, {type(src).__name__})")
    _hook("load", dst, src, coord)


def _check_elem(tile, glob) -> None:
    if tile._dtype.nbytes != glob._dtype.nbytes:
        raise TypeError(
            f"tile element type {tile._dtype.name} and global element type "
            f"{glob._dtype.name} differ in size")


def _store(scope: str, dst, src, coord) -> None:
    b = current_builder()
    mark_kittens(b)
    if isinstance(dst, GlobalHandle):
        if coord is None:
            raise TypeError("store(global, tile, coord) requires a coord tuple")
        if isinstance(src, TensorTile):
            # tensor memory -> global, one accumulator row per thread of the group
            if scope != "warpgroup":
                raise TypeError("store(global, tensor) is a warpgroup operation")
            if dst._dtype.nbytes not in (2, 4) or src._cols % 32:
                raise TypeError("store(global, tensor): 16- or 32-bit global, accumulator columns "
                                "a multiple of 32")
            b.mark_written(dst._expr, kinds=("kittens_global",))
            _stmt(b, f"{NS}::{scope}::store", [dst._expr, src._expr, _coord(coord)])
            _hook("store", dst, src, coord)
            return
        if not isinstance(src, (RegisterTile, SharedTile)):
            raise TypeError(f"kittens.store: cannot store a {type(src).__name__} to global memory")
        if isinstance(src, SharedTile):
            _check_elem(src, dst)
        elif src._layout != "row":
            raise TypeError("store(global, register) needs a row-layout register tile")
        b.mark_written(dst._expr, kinds=("kittens_global",))
        _stmt(b, f"{NS}::{scope}::store", [dst._expr, src._expr, _coord(coord)])
    elif isinstance(dst, SharedTile) and isinstance(src, RegisterTile):
        if coord is not None:
            raise TypeError("store(shared, register) does not take a coord")
        if src._layout != "row":
            raise TypeError("store(shared, register) needs a row-layout register tile")
        _stmt(b, f"{NS}::{scope}::store", [dst._expr, src._expr])
    elif isinstance(dst, SharedTile) and isinstance(src, TensorTile):
        # tensor memory -> shared, one accumulator row per thread of the group
        if scope != "warpgroup" or coord is not None:
            raise TypeError("store(shared, tensor) is a warpgroup operation without a coord")
        if dst._dtype.nbytes != 2 or dst._rows != src._rows or dst._cols > src._cols \
                or dst._cols % 32:
            raise TypeError(
                f"store(shared, tensor): a 16-bit shared tile of the accumulator's {src._rows} rows "
                f"and a multiple of 32 columns up to {src._cols}, got ({dst._rows}, {dst._cols})")
        _stmt(b, f"{NS}::{scope}::store", [dst._expr, src._expr])
    else:
        raise TypeError(
            f"kittens.store: unsupported argument combination "
            f"({type(dst).__name__}, {type(src).__name__})")
    _hook("store", dst, src, coord)


def _swap_layout(scope: str, dst, src) -> None:
    if not (isinstance(dst, RegisterTile) and isinstance(src, RegisterTile)):
        raise TypeError("kittens.swap_layout expects two register tiles")
    if dst._layout == src._layout or dst._dtype.nbytes != 2 or src._dtype != dst._dtype:
        raise TypeError("swap_layout converts a 16-bit register tile between row and column layout")
    b = current_builder()
    mark_kittens(b)
    _stmt(b, f"{NS}::{scope}::swap_layout", [dst._expr, src._expr])
    _hook("swap_layout", dst, src)


def _mma(scope: str, func: str, *args) -> None:
    if not args or not (3 <= len(args) <= 4):
        raise TypeError(f"kittens.{func} expects 3 or 4 register-tile args")
    c, a, bt = args[:3]
    c_in = args[3] if len(args) == 4 else None
    if not all(isinstance(x, RegisterTile) for x in (c, a, bt)):
        raise TypeError(f"kittens.{func} expects register tiles")
    if c_in is None:
        c_in = c
    elif not isinstance(c_in, RegisterTile):
        raise TypeError(f"kittens.{func} c_in must be a RegisterTile")
    b = current_builder()
    mark_kittens(b)
    _stmt(b, f"{NS}::{scope}::{func}", [c._expr, a._expr, bt._expr, c_in._expr])
    _hook(func, c, a, bt, c_in)


_PAIR_FORMS = {"mm_AB": "mm2_AB", "mma_AB": "mma2_AB", "mma_AB_t": "mma2_AB_t", "mm_ABt": "mm2_ABt"}


def _tcgen05(func: str, d, a, bt, sem, ncta=None) -> None:
    if not isinstance(d, TensorTile):
        raise TypeError(f"warpgroup.{func} (tcgen05) d must be a TensorTile")
    if not isinstance(a, SharedTile):
        raise TypeError(f"warpgroup.{func} (tcgen05) a must be a SharedTile")
    if not isinstance(bt, SharedTile):
        raise TypeError(f"warpgroup.{func} (tcgen05) b must be a SharedTile")
    if not isinstance(sem, Semaphore):
        raise TypeError(f"warpgroup.{func} (tcgen05) sem must be a Semaphore")
    pair = (ncta or d._ncta) == 2
    b = current_builder()
    if pair:
        # D's tensor memory must come from a pair allocator; B holds half the
        # columns of D in each CTA
        if d._ncta != 2:
            raise TypeError(f"warpgroup.{_PAIR_FORMS[func]} needs a TensorTile bound to "
                            "tensor_allocator(ncta=2)")
        _mark_pair(b)
        _stmt(b, f"{NS}::warpgroup::{_PAIR_FORMS[func]}", [d._expr, a._expr, bt._expr, sem._expr])
        return
    mark_kittens(b)
    _stmt(b, f"{NS}::warpgroup::{func}", [d._expr, a._expr, bt._expr, sem._expr])


def zero(rt: RegisterTile) -> None:
    """Set every element of a register tile to zero (warp scope)."""
    _zero("warp", rt)


def load(dst, src, coord=None) -> None:
    """Warp-scoped load: ``(shared, global, coord)``, ``(register, shared)``
    or ``(register, global, coord)``; coordinates count tiles."""
    _load("warp", dst, src, coord)


def store(dst, src, coord=None) -> None:
    """Warp-scoped store: ``(global, register|shared, coord)`` or
    ``(shared, register)``."""
    _store("warp", dst, src, coord)


def swap_layout(dst: RegisterTile, src: RegisterTile) -> None:
    """Copy ``src`` into ``dst`` in the other (row <-> column) layout."""
    _swap_layout("warp", dst, src)


def mma_AB(c: RegisterTile, a: RegisterTile, b: RegisterTile, c_in: Optional[RegisterTile] = None):
    """``c = a @ b + c_in`` with ``b`` in column layout (mma.sync)."""
    _mma("warp", "mma_AB", *((c, a, b) if c_in is None else (c, a, b, c_in)))


def mma_AB_t(c: RegisterTile, a: RegisterTile, b: RegisterTile, c_in: Optional[RegisterTile] = None):
    """``c = a @ b^T + c_in`` with ``b`` in row layout (mma.sync)."""
    _mma("warp", "mma_AB_t", *((c, a, b) if c_in is None else (c, a, b, c_in)))


class _WarpgroupNS:
    """Operations of a 4-warp group.  Register tiles are per warp: warp w of
    the group moves rows ``[w*R, (w+1)*R)`` of a shared tile; tcgen05 ops are
    issued by the calling thread."""

    @staticmethod
    def zero(rt):
        _zero("warpgroup", rt)

    @staticmethod
    def load(dst, src, coord=None):
        _load("warpgroup", dst, src, coord)

    @staticmethod
    def store(dst, src, coord=None):
        _store("warpgroup", dst, src, coord)

    @staticmethod
    def swap_layout(dst, src):
        _swap_layout("warp", dst, src)

    @staticmethod
    def mma_AB(*args):
        """Register tiles: ``(c, a, b[, c_in])``; tcgen05: ``(tt_d, st_a, st_b, sem)``
        accumulating ``st_a @ st_b`` into tensor memory and signalling ``sem``
        when the operands have been consumed."""
        if args and isinstance(args[0], TensorTile):
            _tcgen05("mma_AB", *args)
            return
        _mma("warpgroup", "mma_AB", *args)

    @staticmethod
    def mma_AB_t(*args):
        """As ``mma_AB`` with the second operand transposed."""
        if args and isinstance(args[0], TensorTile):
            _tcgen05("mma_AB_t", *args)
            return
        _mma("warpgroup", "mma_AB_t", *args)

    @staticmethod
    def mm_AB(d, a, b, sem):
        """tcgen05 ``d = a @ b`` (overwrites the accumulator)."""
        _tcgen05("mm_AB", d, a, b, sem)

    @staticmethod
    def mm_ABt(d, a, b, sem):
        """tcgen05 ``d = a @ b^T`` (overwrites the accumulator)."""
        _tcgen05("mm_ABt", d, a, b, sem)

    @staticmethod
    def mm2_AB(d, a, b, sem):
        """2-CTA tcgen05 ``d = a @ b`` (M = 256 over the pair), issued by the
        pair leader: ``a`` is each CTA's 128 x K rows, ``b`` its K x N/2
        columns, ``d`` each CTA's 128 x N accumulator; ``sem`` is signalled
        in both CTAs once the operands have been consumed."""
        _tcgen05("mm_AB", d, a, b, sem, ncta=2)

    @staticmethod
    def mma2_AB(d, a, b, sem):
        """2-CTA tcgen05 ``d += a @ b`` (see ``mm2_AB``)."""
        _tcgen05("mma_AB", d, a, b, sem, ncta=2)

    @staticmethod
    def mm2_ABt(d, a, b, sem):
        """2-CTA tcgen05 ``d = a @ b^T`` with ``b`` N/2 x K per CTA."""
        _tcgen05("mm_ABt", d, a, b, sem, ncta=2)

    @staticmethod
    def mma2_AB_t(d, a, b, sem):
        """2-CTA tcgen05 ``d += a @ b^T`` with ``b`` N/2 x K per CTA."""
        _tcgen05("mma_AB_t", d, a, b, sem, ncta=2)

    @staticmethod
    def load_async(dst, src):
        """Tensor memory -> registers: this warp's 32 TMEM lanes into a
        32-row register tile."""
        if not isinstance(dst, RegisterTile):
            raise TypeError("warpgroup.load_async dst must be a RegisterTile")
        if not isinstance(src, TensorTile):
            raise TypeError("warpgroup.load_async src must be a TensorTile")
        b = current_builder()
        mark_kittens(b)
        _stmt(b, f"{NS}::warpgroup::load_async", [dst._expr, src._expr])

    @staticmethod
    def sync(barrier_id: int = 1):
        """Barrier over the 128 threads of this warpgroup."""
        b = current_builder()
        mark_kittens(b)
        _stmt(b, f"{NS}::warpgroup::sync", [ir.Lit(int(barrier_id))])

    @staticmethod
    def laneid() -> Value:
        """This thread's index within its warpgroup (0..127)."""
        b = current_builder()
        mark_kittens(b)
        name = b.fresh_name("wglane")
        b.add_stmt(ir.Decl(name, "int", init=ir.CallExpr(f"{NS}::warpgroup::laneid")))
        return Value(ir.Name(name), dt.int32)


warpgroup = _WarpgroupNS()


class _TmaNS:
    """Tensor Memory Accelerator copies; globals need a tile shape
    (``kittens.Global[dtype, (R, C)]``) that matches the shared tile."""

    @staticmethod
    def expect_bytes(sem: Semaphore, n_bytes) -> None:
        """Arrive on ``sem`` and expect ``n_bytes`` of TMA transfers."""
        if not isinstance(sem, Semaphore):
            raise TypeError("tma.expect_bytes expects a Semaphore")
        b = current_builder()
        _mark_tma(b)
        _stmt(b, f"{NS}::tma::expect_bytes", [sem._expr, to_expr(n_bytes)])

    @staticmethod
    def load_async(dst: SharedTile, src: GlobalHandle, coord: tuple, sem: Semaphore) -> None:
        if not isinstance(dst, SharedTile):
            raise TypeError("tma.load_async dst must be a SharedTile")
        if not isinstance(src, GlobalHandle):
            raise TypeError("tma.load_async src must be a kittens.Global parameter")
        if not isinstance(sem, Semaphore):
            raise TypeError("tma.load_async sem must be a Semaphore")
        _check_tma(dst, src)
        b = current_builder()
        _mark_tma(b)
        _stmt(b, f"{NS}::tma::load_async", [dst._expr, src._expr, _coord(coord), sem._expr])

    @staticmethod
    def store_async(dst: GlobalHandle, src: SharedTile, coord: tuple) -> None:
        if not isinstance(dst, GlobalHandle):
            raise TypeError("tma.store_async dst must be a kittens.Global parameter")
        if not isinstance(src, SharedTile):
            raise TypeError("tma.store_async src must be a SharedTile")
        _check_tma(src, dst)
        b = current_builder()
        _mark_tma(b)
        b.mark_written(dst._expr, kinds=("kittens_global",))
        _stmt(b, f"{NS}::tma::store_async", [dst._expr, src._expr, _coord(coord)])

    @staticmethod
    def store_async_read_wait() -> None:
        """Wait until this thread's TMA stores have read their shared source."""
        b = current_builder()
        _mark_tma(b)
        _stmt(b, f"{NS}::tma::store_async_read_wait", [])


class _TmaPairNS:
    """TMA loads for a CTA pair: each CTA fetches its own tiles into its own
    shared memory (no load is shared between CTAs), and the bytes are counted on
    a semaphore of the CTA ``dst_cta`` — the pair leader, whose MMA reads
    both CTAs' tiles."""

    @staticmethod
    def expect_bytes(sem: Semaphore, n_bytes) -> None:
        """Arrive on this CTA's ``sem`` and expect ``n_bytes`` (both CTAs'
        loads, when it is the leader's)."""
        if not isinstance(sem, Semaphore):
            raise TypeError("tma.pair.expect_bytes expects a Semaphore")
        b = current_builder()
        _mark_tma(b)
        _mark_pair(b)
        _stmt(b, f"{NS}::tma::pair::expect_bytes", [sem._expr, to_expr(n_bytes)])

    @staticmethod
    def load_async(dst: SharedTile, src: GlobalHandle, coord: tuple, sem: Semaphore,
                   dst_cta=0) -> None:
        if not isinstance(dst, SharedTile):
            raise TypeError("tma.pair.load_async dst must be a SharedTile")
        if not isinstance(src, GlobalHandle):
            raise TypeError("tma.pair.load_async src must be a kittens.Global parameter")
        if not isinstance(sem, Semaphore):
            raise TypeError("tma.pair.load_async sem must be a Semaphore")
        _check_tma(dst, src)
        b = current_builder()
        _mark_tma(b)
        _mark_pair(b)
        _stmt(b, f"{NS}::tma::pair::load_async",
              [dst._expr, src._expr, _coord(coord), sem._expr, to_expr(dst_cta)])


_TmaNS.pair = _TmaPairNS()


def _check_tma(tile: SharedTile, glob: GlobalHandle) -> None:
    if glob._tile_shape is None:
        raise TypeError(
            f"TMA on '{glob._param_name}' needs a tile shape: declare it as "
            "kittens.Global[dtype, (rows, cols)]")
    if tuple(glob._tile_shape) != (tile._rows, tile._cols):
        raise TypeError(
            f"TMA tile shape of '{glob._param_name}' is {tuple(glob._tile_shape)} but the shared "
            f"tile is ({tile._rows}, {tile._cols})")
    _check_elem(tile, glob)


tma = _TmaNS()
