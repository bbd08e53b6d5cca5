"""Plumbing shared by the pre-built library kernels: NumPy/DeviceArray
argument binding with the reference's copy-in / launch / synchronise /
copy-back-written semantics (``src/thork/runtime.py:625-700``), around a
C-ABI entry point of libthork_rt.so instead of a traced kernel."""

from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

from .. import dtypes as dt
from .. import runtime as rt


class ArgSpec:
    """One array argument of a library kernel: its name, element type,
    minimum element count and whether the kernel writes it."""

    def __init__(self, name: str, dtype: dt.Dtype, count: int, written: bool = False,
                 overwrites: bool = False, shape: Optional[Tuple[int, ...]] = None):
        self.name = name
        self.dtype = dtype
        self.count = int(count)
        self.written = written
        # the kernel stores every one of the array's elements, so its
        # previous contents need not be copied in
        self.overwrites = overwrites
        self.shape = shape


def _check_array(a, spec: ArgSpec):
    if isinstance(a, rt.DeviceArray):
        if not dt.storage_compatible(a.dtype, spec.dtype):
            raise TypeError(
                f"Argument for pointer parameter '{spec.name}' has dtype {a.dtype}, expected "
                f"{spec.dtype.name}")
        n = int(np.prod(a.shape, dtype=np.int64))
    else:
        if not isinstance(a, np.ndarray):
            raise TypeError(
                f"Argument for pointer parameter '{spec.name}' must be a numpy array, got "
                f"{type(a).__name__}")
        if not dt.storage_compatible(a.dtype, spec.dtype):
            actual = dt.from_numpy(a.dtype)
            raise TypeError(
                f"Argument for pointer parameter '{spec.name}' has dtype {actual.name}, "
                f"expected {spec.dtype.name}")
        if not a.flags["C_CONTIGUOUS"]:
            raise ValueError(f"Argument for pointer parameter '{spec.name}' must be C-contiguous")
        n = a.size
    if n < spec.count:
        raise ValueError(
            f"Argument for '{spec.name}' has {n} elements; the kernel needs {spec.count}")
    if spec.shape is not None and tuple(a.shape) != spec.shape and n != spec.count:
        raise ValueError(f"Argument for '{spec.name}' has shape {tuple(a.shape)}, expected {spec.shape}")
    return a


def run(specs: Sequence[ArgSpec], args: Sequence, launch: Callable[[List[int], Optional[int]], int],
        what: str, stream: Optional["rt.Stream"] = None, sync: bool = True) -> None:
    """Bind ``args`` to device pointers, call ``launch(ptrs, stream_handle)``
    (which returns a thork status code) and copy written host arrays back."""
    rt.get_device()
    if len(args) != len(specs):
        raise TypeError(f"{what} expected {len(specs)} arguments, got {len(args)}")
    s = stream if stream is not None else rt._dispatch_stream()
    owned, ptrs, back = [], [], []
    try:
        for a, spec in zip(args, specs):
            _check_array(a, spec)
            if isinstance(a, rt.DeviceArray):
                ptrs.append(a.ptr)
                continue
            buf = rt.DeviceBuffer(a.nbytes)
            owned.append(buf)
            ptrs.append(buf.ptr)
            if not (spec.overwrites and spec.count == a.size):
                rt.copy_htod(buf.ptr, a, s, sync=False)
            if spec.written:
                back.append((a, buf.ptr))
        rt.check(launch(ptrs, s.handle), what)
        for a, ptr in back:
            rt.copy_dtoh(a, ptr, s, sync=False)
        if sync or back:
            s.synchronize()
    finally:
        for b in owned:
            b.free()


class LibraryKernel:
    """A pre-built kernel with the ``BoundKernel`` call surface:
    ``k(*arrays)`` runs it on NumPy arrays (copied in/out) or DeviceArrays."""

    def __init__(self, name: str, specs: Sequence[ArgSpec], launch, grid=(0, 0, 0),
                 block=(0, 0, 0), source: str = ""):
        self._name = name
        self._specs = list(specs)
        self._launch = launch
        self._grid = tuple(grid)
        self._block = tuple(block)
        self._source = source

    def __call__(self, *args, stream=None, sync: bool = True):
        run(self._specs, args, self._launch, self._name, stream=stream, sync=sync)

    @property
    def name(self) -> str:
        return self._name

    @property
    def grid(self) -> tuple:
        return self._grid

    @property
    def block(self) -> tuple:
        return self._block

    @property
    def cuda_source(self) -> str:
        """Where the kernel comes from (it is compiled ahead of time)."""
        return self._source

    @property
    def source_map(self):
        return {}

    @property
    def specs(self):
        return list(self._specs)


class _Pipe:
    """Per-thread streams for the pipelined host path."""

    def __init__(self):
        self.s_in = rt.Stream()
        self.s_cmp = rt.Stream()
        self.s_out = rt.Stream()


_pipes = {}


def _pipe() -> _Pipe:
    import threading
    key = (threading.get_ident(), rt.get_device())
    p = _pipes.get(key)
    if p is None:
        p = _pipes[key] = _Pipe()
    return p


def chunk_schedule(m: int, chunk_rows: int) -> list:
    """Row counts of the pipelined host path's chunks, summing to ``m``.

    Nothing can be copied out before all of ``b`` and the first chunk of
    ``a`` are on the device, and after the last copy-in only the last
    chunk's kernel and copy-out remain: so the first two chunks are a
    quarter and a half of ``chunk_rows`` and the last three three quarters,
    a quarter and a quarter, with whole chunks between (8192 rows of 8192
    bf16 in 1024-row chunks: 6.00 against 6.11 ms end to end).  Short
    inputs keep equal chunks."""
    if m < 4 * chunk_rows or chunk_rows % 4:
        return [min(chunk_rows, m - r0) for r0 in range(0, m, chunk_rows)]
    q = chunk_rows // 4
    head, tail = [q, 2 * q], [3 * q, q, q]
    mid = m - sum(head) - sum(tail)
    body = [chunk_rows] * (mid // chunk_rows) + ([mid % chunk_rows] if mid % chunk_rows else [])
    return head + body + tail


def run_rows_pipelined(a: np.ndarray, b: np.ndarray, c: np.ndarray, launch_rows, what: str,
                       chunk_rows: int) -> None:
    """``c = f(a, b)`` computed in row chunks of ``a``/``c`` with copy-in,
    compute and copy-out on three streams, so host<->device transfers of one
    chunk overlap the kernel of another.  ``launch_rows(a_ptr, b_ptr, c_ptr,
    rows, stream)`` runs the kernel on ``rows`` rows and returns a status;
    the chunk sizes are ``chunk_schedule(m, chunk_rows)``."""
    ps = _pipe()
    m = a.shape[0]
    bufs = [rt.DeviceBuffer(x.nbytes) for x in (a, b, c)]
    da, db, dc = (x.ptr for x in bufs)
    a_row, c_row = a.nbytes // m, c.nbytes // m
    events = []
    try:
        rt.copy_htod(db, b, ps.s_in, sync=False)
        r1 = 0
        for rows in chunk_schedule(m, chunk_rows):
            r0, r1 = r1, r1 + rows
            ev_in, ev_done = rt.Event(), rt.Event()
            events += [ev_in, ev_done]
            rt.copy_htod(da + r0 * a_row, a[r0:r1], ps.s_in, sync=False)
            ev_in.record(ps.s_in)
            ps.s_cmp.wait(ev_in)
            rt.check(launch_rows(da + r0 * a_row, db, dc + r0 * c_row, r1 - r0, ps.s_cmp.handle), what)
            ev_done.record(ps.s_cmp)
            ps.s_out.wait(ev_done)
            rt.copy_dtoh(c[r0:r1], dc + r0 * c_row, ps.s_out, sync=False)
        ps.s_out.synchronize()
    finally:
        for e in events:
            e.close()
        for x in bufs:
            x.free()


def is_host(*arrays) -> bool:
    return all(isinstance(x, np.ndarray) for x in arrays)
