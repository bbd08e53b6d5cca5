"""``@tk.jit``: trace once, compile with NVRTC for sm_100a, launch on NumPy
arrays with automatic copy-in / copy-back.

Same surface as the reference's ``src/thork/jit.py``: ``JittedKernel``
(``jit.py:41-191``) with ``kernel[grid, block](*args)``, ``.bind``,
``.compile_for_arch``, ``.cuda_source`` and ``.source_map``; ``BoundKernel``
(``jit.py:236-270``).  Differences: tile (``kittens``) kernels compile through
NVRTC as well (no nvcc host launcher), request only the dynamic shared memory
their tiles need, and ``compile_for_arch`` works for every kernel.
"""

import inspect
from typing import Callable, Optional

from . import ir
from . import runtime
from . import tracer as _tr
from .codegen import emit_kernel
from .tracer import KernelBuilder, Pointer, Value, Vector
from .types import DevicePointerSpec, KittensGlobalSpec, spec_from_annotation

_SUPPORTED_ARCHES = ("100a", "sm_100a", "100", "sm_100")


class JittedKernel:
    """A function decorated with ``@tk.jit``."""

    def __init__(self, fn: Callable, name: Optional[str] = None):
        self._fn = fn
        self.name = name or fn.__name__
        self._sig = inspect.signature(fn)
        self._builder: Optional[KernelBuilder] = None
        self._source: Optional[str] = None
        self._source_map: Optional[dict] = None
        self._module: Optional[runtime.Module] = None
        self._func: Optional[int] = None

    # -- tracing
    def _trace(self) -> KernelBuilder:
        b = KernelBuilder(self.name)
        args = []
        for pname, p in self._sig.parameters.items():
            if p.kind in (inspect.Parameter.VAR_POSITIONAL, inspect.Parameter.VAR_KEYWORD):
                raise TypeError(f"Kernel '{self.name}': *args/**kwargs not supported")
            if p.annotation is inspect.Parameter.empty:
                raise TypeError(
                    f"Kernel '{self.name}': parameter '{pname}' is missing a type annotation")
            spec = spec_from_annotation(p.annotation, self.name, pname)
            if isinstance(spec, DevicePointerSpec):
                b.params.append(ir.Param(pname, "pointer", spec.dtype))
                args.append(Pointer(ir.Name(pname), spec.dtype, b))
            elif isinstance(spec, KittensGlobalSpec):
                from .kittens import GlobalHandle, mark_kittens
                b.params.append(ir.Param(pname, "kittens_global", spec.dtype,
                                         tile_shape=spec.tile_shape))
                mark_kittens(b)
                args.append(GlobalHandle(ir.Name(pname), spec.dtype, b, spec.tile_shape))
            else:
                kind = "attribute" if spec.attribute is not None else "constant"
                b.params.append(ir.Param(pname, kind, spec.dtype, cuda_name=spec.cuda_name,
                                         vec_size=spec.vec_size, attribute=spec.attribute))
                if spec.vec_size > 1:
                    args.append(Vector(ir.Name(pname), spec.dtype, spec.vec_size))
                else:
                    args.append(Value(ir.Name(pname), spec.dtype))
        token = _tr._active.set(b)
        try:
            self._fn(*args)
        finally:
            _tr._active.reset(token)
        if b.uses_kittens:
            from .kittens import finalize
            finalize(b)
        return b

    def _ensure_traced(self) -> None:
        if self._source is None:
            self._builder = self._trace()
            self._source, self._source_map = emit_kernel(self._builder)

    def _ensure_compiled(self) -> None:
        if self._func is not None:
            return
        self._ensure_traced()
        self._module = runtime.compile_source(self._source, source_map=self._source_map)
        self._func = self._module.function(self.name)
        smem = self.dynamic_smem
        if smem > 48 * 1024:
            runtime.check(runtime.lib().thork_function_set_max_dynamic_smem(self._func, smem),
                          "set max dynamic smem")

    @property
    def dynamic_smem(self) -> int:
        """Dynamic shared memory this kernel's tile allocations need."""
        self._ensure_traced()
        return int(getattr(self._builder, "dynamic_smem", 0))

    # -- launching
    def __getitem__(self, dispatch_spec) -> "_Launcher":
        """``kernel[grid, block]``, or ``kernel[grid, block, cluster]`` for a
        thread-block-cluster launch (2-CTA tile kernels use ``(2, 1, 1)``)."""
        if not (isinstance(dispatch_spec, tuple) and len(dispatch_spec) in (2, 3)):
            raise TypeError(
                f"Kernel must be subscripted with (grid_size, block_size), got {dispatch_spec!r}")
        return _Launcher(self, *dispatch_spec)

    def bind(self, grid, block, cluster=None) -> "BoundKernel":
        """A callable with ``grid``/``block`` (and ``cluster``) baked in."""
        return BoundKernel(self, grid, block, cluster)

    @property
    def cluster_ctas(self) -> int:
        """CTAs per cluster the kernel's tile operations need (2 for
        cluster-pair tensor-core operations, else 1)."""
        self._ensure_traced()
        return int(getattr(self._builder, "tk_cluster", 1))

    def compile_for_arch(self, arch: str) -> None:
        """Trace and compile (NVRTC, no launch) for ``arch``; only sm_100a
        targets are supported ("100a", "100" and the sm_ spellings all build
        sm_100a code).  Raises on compile failure."""
        if str(arch) not in _SUPPORTED_ARCHES:
            raise ValueError(f"thork_b200 compiles for sm_100a only, got arch {arch!r}")
        b = self._trace()
        src, smap = emit_kernel(b)
        runtime.nvrtc_compile(src, source_map=smap)

    @property
    def cuda_source(self) -> str:
        self._ensure_traced()
        return self._source

    @property
    def source_map(self) -> Optional[dict]:
        """Generated line (1-based) -> (python file, line)."""
        self._ensure_traced()
        return self._source_map

    @property
    def params(self):
        self._ensure_traced()
        return list(self._builder.params)


def _dims(v) -> tuple:
    t = tuple(int(x) for x in v)
    if len(t) != 3:
        raise TypeError(f"grid/block must have 3 components, got {v!r}")
    return t


class _Launcher:
    __slots__ = ("_kernel", "_grid", "_block", "_cluster", "_prepare")

    def __init__(self, kernel: JittedKernel, grid, block, cluster=None):
        self._kernel = kernel
        self._grid = _dims(grid)
        self._block = _dims(block)
        self._cluster = _dims(cluster) if cluster is not None else None
        self._prepare = False

    def prepare(self, *args) -> "runtime.PreparedLaunch":
        """Pack device-resident arguments once; ``.launch(stream)`` then queues
        the kernel asynchronously (no copies, no synchronisation)."""
        self._prepare = True
        try:
            return self(*args)
        finally:
            self._prepare = False

    def __call__(self, *args):
        k = self._kernel
        need = k.cluster_ctas  # traces the kernel; checked before any compile or launch
        cl = self._cluster or (1, 1, 1)
        if need > 1 and cl != (need, 1, 1):
            raise ValueError(
                f"Kernel '{k.name}' uses cluster-pair tile operations; launch it as "
                f"kernel[grid, block, ({need}, 1, 1)] (got cluster {cl})")
        if cl[0] * cl[1] * cl[2] > 1 and any(g % c for g, c in zip(self._grid, cl)):
            raise ValueError(f"grid {self._grid} is not a multiple of the cluster {cl}")
        k._ensure_compiled()
        if getattr(self, "_prepare", False):
            return runtime.PreparedLaunch(k._func, k._builder.params, args, self._grid, self._block,
                                          k.dynamic_smem, uses_status=k._builder.uses_status,
                                          cluster=self._cluster)
        runtime.dispatch(k._func, k._builder.params, args, self._grid, self._block,
                         shared_mem_bytes=k.dynamic_smem, uses_status=k._builder.uses_status,
                         name=k.name, cluster=self._cluster)


def jit(fn: Callable) -> JittedKernel:
    """Decorator: turn a Python function into a CUDA kernel (traced on first
    launch, compiled with NVRTC for sm_100a)."""
    return JittedKernel(fn)


class BoundKernel:
    """A JittedKernel with grid and block bound; call it with the pointer and
    constant arguments."""

    __slots__ = ("_kernel", "_grid", "_block", "_cluster")

    def __init__(self, kernel, grid, block, cluster=None):
        self._kernel = kernel
        self._grid = tuple(int(x) for x in grid)
        self._block = tuple(int(x) for x in block)
        self._cluster = tuple(int(x) for x in cluster) if cluster is not None else None

    def _launcher(self) -> "_Launcher":
        if self._cluster is None:
            return self._kernel[self._grid, self._block]
        return self._kernel[self._grid, self._block, self._cluster]

    def __call__(self, *args):
        self._launcher()(*args)

    def prepare(self, *args) -> "runtime.PreparedLaunch":
        """See ``_Launcher.prepare``: device-resident arguments packed once
        for asynchronous launches."""
        return self._launcher().prepare(*args)

    @property
    def cuda_source(self) -> str:
        return self._kernel.cuda_source

    @property
    def source_map(self):
        return self._kernel.source_map

    @property
    def grid(self) -> tuple:
        return self._grid

    @property
    def block(self) -> tuple:
        return self._block

    @property
    def name(self) -> str:
        return self._kernel.name
