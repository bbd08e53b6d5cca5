"""Kernels written against the thork API, used by both implementations.

``build(tk)`` defines the kernels with whichever package is passed as ``tk``
(thork_b200 in the tests; the reference ``thork`` in
``tests/golden/make_golden.py``), so the two traces can be compared: same
parameter list, kinds and ``written`` flags (which decide copy-back).  Each
kernel exercises one part of the tracing surface.
"""


def build(tk):
    f32 = tk.dt.float32
    u32 = tk.dt.uint32
    P = tk.DevicePointer
    kernels = {}

    @tk.jit
    def vec_add(out: P[f32], a: P[f32], b: P[f32],
                bid: tk.Uint[tk.BlockIdx], tid: tk.Uint[tk.ThreadIdx], bdm: tk.Uint[tk.BlockDim]):
        i = bid * bdm + tid
        out[i] = a[i] + b[i]
    kernels["vec_add"] = vec_add

    @tk.jit
    def saxpy_strided(y: P[f32], x: P[f32], alpha: tk.Uint, n: tk.Uint,
                      bid: tk.Uint[tk.BlockIdx], tid: tk.Uint[tk.ThreadIdx],
                      bdm: tk.Uint[tk.BlockDim], gdm: tk.Uint[tk.GridDim]):
        for i in tk.range(bid * bdm + tid, n, bdm * gdm):
            y[i] = y[i] + tk.cast(alpha, f32) * x[i]
    kernels["saxpy_strided"] = saxpy_strided

    @tk.jit
    def row_dot(out: P[f32], a: P[f32], b: P[f32], k: tk.Uint, n: tk.Uint,
                blk: tk.Uint2[tk.BlockIdx], thr: tk.Uint2[tk.ThreadIdx], dim: tk.Uint2[tk.BlockDim]):
        r = blk.y * dim.y + thr.y
        c = blk.x * dim.x + thr.x
        acc = tk.local(f32, 0.0)
        for kk in tk.range(k):
            acc += a[r * k + kk] * b[kk * n + c]
        out[r * n + c] = acc
    kernels["row_dot"] = row_dot

    @tk.jit
    def tiled_mm(out: P[f32], a: P[f32], b: P[f32], m: tk.Uint, n: tk.Uint, k: tk.Uint,
                 blk: tk.Uint2[tk.BlockIdx], thr: tk.Uint2[tk.ThreadIdx]):
        T = 16
        sa = tk.shared(f32, (T, T))
        sb = tk.shared(f32, (T, T))
        r = blk.y * T + thr.y
        c = blk.x * T + thr.x
        acc = tk.local(f32, 0.0)
        for k0 in tk.range(0, k, T):
            sa[thr.y, thr.x] = a[r * k + k0 + thr.x]
            sb[thr.y, thr.x] = b[(k0 + thr.y) * n + c]
            tk.syncthreads()
            for kk in tk.range(T):
                acc += sa[thr.y, kk] * sb[kk, thr.x]
            tk.syncthreads()
        out[r * n + c] = acc
    kernels["tiled_mm"] = tiled_mm

    @tk.jit
    def softplus(out: P[f32], a: P[f32],
                 bid: tk.Uint[tk.BlockIdx], tid: tk.Uint[tk.ThreadIdx], bdm: tk.Uint[tk.BlockDim]):
        i = bid * bdm + tid
        x = a[i]
        out[i] = tk.log(1.0 + tk.exp(x)) + tk.fmax(x, 0.0) * 0.0
    kernels["softplus"] = softplus

    @tk.jit
    def bincount(counts: P[u32], values: P[u32], nbins: tk.Uint,
                 bid: tk.Uint[tk.BlockIdx], tid: tk.Uint[tk.ThreadIdx], bdm: tk.Uint[tk.BlockDim]):
        v = values[bid * bdm + tid]
        tk.atomic_add(counts, v % nbins, 1)
    kernels["bincount"] = bincount

    @tk.jit
    def warp_dot(out: P[f32], a: P[f32], b: P[f32], k: tk.Uint,
                 bid: tk.Uint[tk.BlockIdx], lane: tk.Uint[tk.LaneId], wsz: tk.Uint[tk.WarpSize]):
        part = tk.local(f32, 0.0)
        for kk in tk.range(lane, k, wsz):
            part += a[bid * k + kk] * b[bid * k + kk]
        total = tk.warp_sum(part)
        with tk.if_(lane == 0):
            out[bid] = total
    kernels["warp_dot"] = warp_dot

    @tk.device_fn
    def halley_cbrt(x: f32) -> f32:
        g = tk.local(f32, x)
        it = tk.local(u32, 0)
        with tk.while_(it < 40):
            g3 = g * g * g
            nxt = g * (g3 + 2.0 * x) / (2.0 * g3 + x)
            with tk.if_(tk.fabs(nxt - g) < 1e-7):
                tk.break_()
            g.assign(nxt)
            it += 1
        return g

    @tk.jit
    def cbrt_pos(out: P[f32], a: P[f32],
                 bid: tk.Uint[tk.BlockIdx], tid: tk.Uint[tk.ThreadIdx], bdm: tk.Uint[tk.BlockDim]):
        i = bid * bdm + tid
        x = a[i]
        with tk.if_(x <= 0.0) as br:
            out[i] = 0.0
        with br.else_():
            out[i] = halley_cbrt(x)
    kernels["cbrt_pos"] = cbrt_pos

    @tk.jit
    def read_only(a: P[f32], b: P[f32], tid: tk.Uint[tk.ThreadIdx]):
        x = a[tid] + b[tid]
        tk.syncthreads()
    kernels["read_only"] = read_only

    return kernels


def build_tiles(tk):
    """Tile-API kernels (trace only): parameter kinds and written flags."""
    G = tk.kittens.Global
    bf = tk.dt.bfloat16
    kernels = {}

    @tk.jit
    def copy_tile(A: G[bf], B: G[bf]):
        s = tk.kittens.st_bf(32, 32)
        tk.kittens.load(s, A, (0, 0))
        tk.kittens.store(B, s, (0, 0))
    kernels["copy_tile"] = copy_tile

    @tk.jit
    def tma_copy(A: G[bf, (64, 64)], B: G[bf, (64, 64)], tid: tk.Uint[tk.ThreadIdx],
                 bid: tk.Uint2[tk.BlockIdx]):
        s = tk.kittens.st_bf(64, 64)
        sem = tk.kittens.semaphore()
        with tk.if_(tid == 0):
            tk.kittens.init_semaphore(sem, 0, 1)
        tk.syncthreads()
        with tk.if_(tid == 0):
            tk.kittens.tma.expect_bytes(sem, 64 * 64 * 2)
            tk.kittens.tma.load_async(s, A, (bid.y, bid.x), sem)
        tk.kittens.wait(sem, 0)
        with tk.if_(tid == 0):
            tk.kittens.tma.store_async(B, s, (bid.y, bid.x))
            tk.kittens.tma.store_async_read_wait()
    kernels["tma_copy"] = tma_copy
    return kernels
