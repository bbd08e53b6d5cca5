"""thork_b200.kernels — pre-built kernels with launch geometry chosen for you
(reference ``src/thork/kernels/__init__.py``)::

    mm = tk.kernels.matmul(4096, 4096, 4096, dtype=tk.dt.bfloat16)
    mm(C, A, B)

    add = tk.kernels.matrix_add((1024, 1024))
    add(C, A, B)

    tm = tk.kernels.tile_matmul(4096, 4096, 4096, ncta=2)   # written in tk.kittens
    tm(C, A, B)
"""

from .matmul import matmul
from .matrix_add import matrix_add
from .tile_matmul import tile_matmul

__all__ = ["matmul", "matrix_add", "tile_matmul"]
