"""Tile-API kernels (the tk.kittens front end), written for these tests:
a register-tile mma.sync matmul, a TMA-fed one, and a tcgen05/TMEM one.
``build(tk, ...)`` returns jitted kernels; shapes are module constants."""


def regtile_matmul(tk, BLOCK=32):
    """One warp per BLOCK x BLOCK output tile: shared tiles filled by warp
    loads, register tiles, swap_layout, warp mma_AB, direct global store."""
    G = tk.kittens.Global
    bf = tk.dt.bfloat16

    @tk.jit
    def regtile_mm(A: G[bf], B: G[bf], C: G[bf], K: tk.Uint, blk: tk.Uint2[tk.BlockIdx]):
        a_s = tk.kittens.st_bf(BLOCK, BLOCK)
        b_s = tk.kittens.st_bf(BLOCK, BLOCK)
        a_r = tk.kittens.rt_bf(BLOCK, BLOCK)
        b_r = tk.kittens.rt_bf(BLOCK, BLOCK)
        b_c = tk.kittens.rt_bf_col(BLOCK, BLOCK)
        acc = tk.kittens.rt_fl(BLOCK, BLOCK)
        tk.kittens.zero(acc)
        for kt in tk.range(K // BLOCK):
            tk.kittens.load(a_s, A, (blk.y, kt))
            tk.kittens.load(b_s, B, (kt, blk.x))
            tk.syncwarp()
            tk.kittens.load(a_r, a_s)
            tk.kittens.load(b_r, b_s)
            tk.kittens.swap_layout(b_c, b_r)
            tk.syncwarp()
            tk.kittens.mma_AB(acc, a_r, b_c, acc)
        tk.kittens.store(C, acc, (blk.y, blk.x))

    return regtile_mm


def tma_matmul(tk, TM=64, TN=64, TK=32):
    """TMA loads into swizzled shared tiles on one semaphore, warp mma_AB,
    shared staging and a TMA store."""
    G = tk.kittens.Global
    bf = tk.dt.bfloat16

    @tk.jit
    def tma_mm(A: G[bf, (TM, TK)], B: G[bf, (TK, TN)], C: G[bf, (TM, TN)], K: tk.Uint,
               blk: tk.Uint2[tk.BlockIdx], tid: tk.Uint[tk.ThreadIdx]):
        a_s = tk.kittens.st_bf(TM, TK)
        b_s = tk.kittens.st_bf(TK, TN)
        c_s = tk.kittens.st_bf(TM, TN)
        arrived = tk.kittens.semaphore()
        with tk.if_(tid == 0):
            tk.kittens.init_semaphore(arrived, 0, 1)
        tk.syncthreads()
        a_r = tk.kittens.rt_bf(TM, TK)
        b_r = tk.kittens.rt_bf(TK, TN)
        b_c = tk.kittens.rt_bf_col(TK, TN)
        acc = tk.kittens.rt_fl(TM, TN)
        tk.kittens.zero(acc)
        phase = tk.local(tk.dt.int32, 0)
        for kt in tk.range(K // TK):
            with tk.if_(tid == 0):
                tk.kittens.tma.expect_bytes(arrived, (TM * TK + TK * TN) * 2)
                tk.kittens.tma.load_async(a_s, A, (blk.y, kt), arrived)
                tk.kittens.tma.load_async(b_s, B, (kt, blk.x), arrived)
            tk.kittens.wait(arrived, phase)
            phase ^= 1
            tk.kittens.load(a_r, a_s)
            tk.kittens.load(b_r, b_s)
            tk.kittens.swap_layout(b_c, b_r)
            tk.kittens.mma_AB(acc, a_r, b_c, acc)
            tk.syncthreads()
        tk.kittens.store(c_s, acc)
        tk.syncthreads()
        with tk.if_(tid == 0):
            tk.kittens.tma.store_async(C, c_s, (blk.y, blk.x))
            tk.kittens.tma.store_async_read_wait()

    return tma_mm


def tcgen05_matmul(tk, TM=128, TN=128, TK=64, WARPS=4):
    """TMA loads, tcgen05 mm_AB/mma_AB into a TMEM accumulator, commit,
    TMEM -> registers per warp, shared staging, TMA store (128 threads)."""
    G = tk.kittens.Global
    bf = tk.dt.bfloat16

    @tk.jit
    def umma_mm(A: G[bf, (TM, TK)], B: G[bf, (TK, TN)], D: G[bf, (TM, TN)], K: tk.Uint,
                N: tk.Uint, bid: tk.Uint[tk.BlockIdx], tid: tk.Uint[tk.ThreadIdx]):
        lane = tk.kittens.warpgroup.laneid()
        grid_n = N // TN
        bm = bid // grid_n
        bn = bid % grid_n
        a_s = tk.kittens.st_bf(TM, TK)
        b_s = tk.kittens.st_bf(TK, TN)
        d_s = tk.kittens.st_bf(TM, TN)
        arrived = tk.kittens.semaphore()
        consumed = tk.kittens.semaphore()
        done = tk.kittens.semaphore()
        with tk.if_(tid == 0):
            tk.kittens.init_semaphore(arrived, 0, 1)
            tk.kittens.init_semaphore(consumed, 1, 0)
            tk.kittens.init_semaphore(done, 0, 1)
        tk.syncthreads()
        tm = tk.kittens.tensor_allocator()
        acc = tk.kittens.tt_fl(TM, TN)
        with tk.if_(lane == 0):
            tk.kittens.tensor_alloc(acc, tm, 0)
        tk.kittens.warpgroup.sync(1)
        phase = tk.local(tk.dt.int32, 0)
        for it in tk.range(K // TK):
            with tk.if_(tid == 0):
                tk.kittens.wait(consumed, phase ^ 1)
                tk.kittens.tma.expect_bytes(arrived, (TM * TK + TK * TN) * 2)
                tk.kittens.tma.load_async(a_s, A, (bm, it), arrived)
                tk.kittens.tma.load_async(b_s, B, (it, bn), arrived)
            tk.kittens.wait(arrived, phase)
            phase ^= 1
            with tk.if_(lane == 0):
                with tk.if_(it == 0) as first:
                    tk.kittens.warpgroup.mm_AB(acc, a_s, b_s, consumed)
                with first.else_():
                    tk.kittens.warpgroup.mma_AB(acc, a_s, b_s, consumed)
        with tk.if_(lane == 0):
            tk.kittens.tcgen05_commit(done)
        tk.kittens.wait(done, 0)
        d_r = tk.kittens.rt_bf(TM // WARPS, TN)
        tk.kittens.warpgroup.load_async(d_r, acc)
        tk.kittens.tensor_load_wait()
        tk.kittens.warpgroup.sync(1)
        tk.kittens.warpgroup.store(d_s, d_r)
        tk.kittens.warpgroup.sync(1)
        with tk.if_(lane == 0):
            tk.kittens.tma.store_async(D, d_s, (bm, bn))
            tk.kittens.tma.store_async_read_wait()

    return umma_mm
