"""thork_b200.kernels — pre-built kernels with launch geometry chosen for you
(reference ``src/thork/kernels/__init__.py``)::

    mm = tk.kernels.matmul(4096, 4096, 4096, dtype=tk.dt.bfloat16)
    mm(C, A, B)

    add = tk.kernels.matrix_add((1024, 1024))
    add(C, A, B)
"""

from .matmul import matmul
from .matrix_add import matrix_add

__all__ = ["matmul", "matrix_add"]
