"""``tk.kernels.matmul(M, N, K, dtype)``: ``out = A @ B`` (row-major).

Drop-in for the reference's ``src/thork/kernels/matmul.py:17-71`` (a 16x16
shared-memory SIMT kernel, float32 only).  Routing by dtype:

* ``float32``: a traced shared-memory-tiled SIMT kernel (API parity; M, N, K
  multiples of 16 like the reference).
* ``bfloat16``: the tcgen05 GEMM ``thork_gemm_bf16`` (TMA, mbarrier pipeline,
  TMEM accumulators), or for M <= 256 the swap-AB decode kernel
  ``thork_skinny_gemm_bf16``.  Output bf16, fp32 accumulation.
* ``float8_e4m3``: ``thork_gemm_e4m3``; call as ``k(out, A, B, scale_a,
  scale_b)`` with per-tensor scales, output bf16 = scale_a*scale_b*(A@B).

Arguments are ``(out, A, B)`` like the reference.  bf16 arrays may be
``ml_dtypes.bfloat16`` or raw ``uint16``; e4m3 arrays ``float8_e4m3fn`` or
``uint8``.
"""

from .. import dtypes as dt
from .. import runtime as rt
from ..jit import jit
from ..tracer import local, range as tk_range, shared, syncthreads
from ..types import BlockIdx, DevicePointer, ThreadIdx, Uint2
from ._library import ArgSpec, LibraryKernel, _check_array, is_host, run, run_rows_pipelined

_TILE = 16


def _simt_matmul(M: int, N: int, K: int, dtype: dt.Dtype):
    if M % _TILE or N % _TILE or K % _TILE:
        raise ValueError(
            f"matmul: M, N, K must all be multiples of {_TILE}; got M={M}, N={N}, K={K}")

    @jit
    def matmul_kernel(
        out: DevicePointer[dtype],
        A: DevicePointer[dtype],
        B: DevicePointer[dtype],
        bid: Uint2[BlockIdx],
        tid: Uint2[ThreadIdx],
    ):
        a_s = shared(dtype, (_TILE, _TILE))
        b_s = shared(dtype, (_TILE, _TILE))
        r = bid.y * _TILE + tid.y
        c = bid.x * _TILE + tid.x
        acc = local(dtype, 0.0)
        for k0 in tk_range(0, K, _TILE):
            a_s[tid.y, tid.x] = A[r * K + k0 + tid.x]
            b_s[tid.y, tid.x] = B[(k0 + tid.y) * N + c]
            syncthreads()
            for kk in tk_range(_TILE):
                acc += a_s[tid.y, kk] * b_s[kk, tid.x]
            syncthreads()
        out[r * N + c] = acc

    return matmul_kernel.bind(grid=(N // _TILE, M // _TILE, 1), block=(_TILE, _TILE, 1))


def _chunk_rows(m: int) -> int:
    """Row-chunk size of the pipelined host path (multiples of 256 rows)."""
    return max(256, ((m // 8) + 255) // 256 * 256)


def _pipelinable(specs, args, m: int) -> bool:
    """Host NumPy operands large enough that overlapping their transfers pays."""
    if m < 1024 or not is_host(*args):
        return False
    for a, spec in zip(args, specs):
        _check_array(a, spec)
        if a.size != spec.count:
            return False
    return True


class _GemmKernel(LibraryKernel):
    """A GEMM whose NumPy-argument calls stream row chunks through
    copy-in / tcgen05 GEMM / copy-out on three streams."""

    def __init__(self, name, specs, launch, rows_launch, m, source=""):
        super().__init__(name, specs, launch, source=source)
        self._rows = rows_launch
        self._m = m

    def __call__(self, *args, stream=None, sync: bool = True):
        if stream is None and len(args) == 3 and _pipelinable(self._specs, args, self._m):
            rt.get_device()
            out, a, b = args
            run_rows_pipelined(a, b, out, self._rows, self._name, _chunk_rows(self._m))
            return
        super().__call__(*args, stream=stream, sync=sync)


def matmul(M: int, N: int, K: int, dtype: dt.Dtype = dt.float32, variant: str = "auto",
           static_weights: bool = False):
    """Return a kernel ``k(out, A, B)`` for ``out[M,N] = A[M,K] @ B[K,N]``.

    ``variant``: ``"auto"``, ``"gemm"`` (128x256 tcgen05 tiles, one CTA),
    ``"gemm2"`` (256x256 tiles on a 2-CTA cluster), ``"gemm_sk"`` (128x256
    tiles, stream-K: equal shares of the k-loop per SM, split tiles summed
    in a fixup) or, bf16 only, ``"skinny"`` (swap-AB, M <= 256).  ``static_weights`` (skinny): B is
    written by no earlier kernel on the stream (decode weights), so the
    kernel may start fetching it before the previous kernel has finished.
    """
    M, N, K = int(M), int(N), int(K)
    if dtype == dt.float32:
        return _simt_matmul(M, N, K, dtype)
    if M <= 0 or N <= 0 or K <= 0:
        raise ValueError(f"matmul: dimensions must be positive; got M={M}, N={N}, K={K}")
    if dtype == dt.bfloat16:
        if K % 8 or N % 8:
            raise ValueError(f"matmul(bf16): K and N must be multiples of 8; got N={N}, K={K}")
        if variant == "auto":
            variant = "skinny" if M <= 256 else "gemm_auto"
        specs = [ArgSpec("out", dt.bfloat16, M * N, written=True, overwrites=True),
                 ArgSpec("A", dt.bfloat16, M * K), ArgSpec("B", dt.bfloat16, K * N)]
        if variant == "skinny":
            if M > 256:
                raise ValueError(f"matmul(bf16, skinny): M must be <= 256, got {M}")

            flags = 1 if static_weights else 0  # THORK_SKINNY_W_STATIC

            def launch(p, s):
                return rt.lib().thork_skinny_gemm_bf16_ex(p[1], p[2], p[0], M, N, K, flags, s)

            name = "skinny_gemm_bf16"
        elif variant in ("gemm", "gemm2", "gemm_sk", "gemm_auto"):
            code = {"gemm_auto": 0, "gemm": 1, "gemm2": 2, "gemm_sk": 3}[variant]

            def launch(p, s):
                return rt.lib().thork_gemm_bf16(p[1], p[2], p[0], M, N, K, code, s)

            def rows(a, b, c, m, s):
                return rt.lib().thork_gemm_bf16(a, b, c, m, N, K, code, s)

            return _GemmKernel("gemm_bf16", specs, launch, rows, M,
                               source="libthork_rt.so: thork_gemm_bf16")
        else:
            raise ValueError(f"matmul: unknown variant {variant!r}")
        return LibraryKernel(name, specs, launch, source=f"libthork_rt.so: thork_{name}")
    if dtype == dt.float8_e4m3:
        if K % 16 or N % 16:
            raise ValueError(f"matmul(e4m3): K and N must be multiples of 16; got N={N}, K={K}")
        specs = [ArgSpec("out", dt.bfloat16, M * N, written=True, overwrites=True),
                 ArgSpec("A", dt.float8_e4m3, M * K), ArgSpec("B", dt.float8_e4m3, K * N)]

        code = {"auto": 0, "gemm": 1, "gemm2": 2, "gemm_sk": 3}.get(variant)
        if code is None:
            raise ValueError(f"matmul: unknown variant {variant!r}")

        class _Fp8(LibraryKernel):
            def __call__(self, out, A, B, scale_a=1.0, scale_b=1.0, stream=None, sync=True):
                sa, sb = float(scale_a), float(scale_b)

                def launch(p, s):
                    return rt.lib().thork_gemm_e4m3(p[1], p[2], p[0], M, N, K, sa, sb, code, s)

                def rows(a, b, c, m, s):
                    return rt.lib().thork_gemm_e4m3(a, b, c, m, N, K, sa, sb, code, s)

                if stream is None and _pipelinable(self._specs, (out, A, B), M):
                    rt.get_device()
                    run_rows_pipelined(A, B, out, rows, self._name, _chunk_rows(M))
                    return
                run(self._specs, (out, A, B), launch, self._name, stream=stream, sync=sync)

        return _Fp8("gemm_e4m3", specs, None, source="libthork_rt.so: thork_gemm_e4m3")
    raise TypeError(f"matmul: unsupported dtype {dtype!r}")
