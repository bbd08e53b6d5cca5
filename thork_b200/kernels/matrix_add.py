"""``tk.kernels.matrix_add(shape, dtype)``: elementwise ``out = A + B``.

Drop-in for the reference's ``src/thork/kernels/matrix_add.py:15-52``.  For
float32 (the benchmarked case) the call goes to the hand-written
``thork_matrix_add_f32`` (128-bit vectorised, grid-stride, streaming
loads/stores) in libthork_rt.so; other dtypes use a traced grid-stride
kernel compiled by NVRTC.  Arrays are treated as flat buffers of
``prod(shape)`` elements, as in the reference.
"""

import math
from typing import Sequence

from .. import dtypes as dt
from .. import runtime as rt
from ..jit import BoundKernel, jit
from ..tracer import range as tk_range
from ..types import BlockDim, BlockIdx, DevicePointer, GridDim, ThreadIdx, Uint
from ._library import ArgSpec, LibraryKernel


def matrix_add(shape: Sequence[int], dtype: dt.Dtype = dt.float32):
    """Return a kernel ``k(out, A, B)`` computing ``out = A + B``."""
    n = int(math.prod(shape))
    if n <= 0:
        raise ValueError(f"matrix_add: shape {tuple(shape)!r} has zero elements")
    if dtype == dt.float32:
        specs = [ArgSpec("out", dtype, n, written=True, overwrites=True),
                 ArgSpec("A", dtype, n), ArgSpec("B", dtype, n)]

        def launch(ptrs, stream):
            return rt.lib().thork_matrix_add_f32(ptrs[0], ptrs[1], ptrs[2], n, stream)

        return LibraryKernel("matrix_add_f32", specs, launch, grid=(0, 0, 0), block=(256, 1, 1),
                             source="libthork_rt.so: thork_matrix_add_f32 (add_f32_v4_kernel)")

    @jit
    def matrix_add_kernel(
        out: DevicePointer[dtype],
        A: DevicePointer[dtype],
        B: DevicePointer[dtype],
        count: Uint,
        bid: Uint[BlockIdx],
        tid: Uint[ThreadIdx],
        bdm: Uint[BlockDim],
        gdm: Uint[GridDim],
    ):
        for i in tk_range(bid * bdm + tid, count, bdm * gdm):
            out[i] = A[i] + B[i]

    block = 256
    grid = min((n + block - 1) // block, 148 * 8)
    bound = BoundKernel(matrix_add_kernel, (grid, 1, 1), (block, 1, 1))

    class _Add:
        def __call__(self, out, A, B):
            bound(out, A, B, n)

        grid = bound.grid
        block = bound.block
        name = bound.name

        @property
        def cuda_source(self):
            return bound.cuda_source

        @property
        def source_map(self):
            return bound.source_map

    return _Add()
