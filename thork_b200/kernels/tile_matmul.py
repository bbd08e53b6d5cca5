"""``tk.kernels.tile_matmul(M, N, K, ncta=1)``: ``C = A @ B`` in bf16 (fp32
accumulation in tensor memory), written in the traced tile DSL itself.

The reference's pre-built kernels are ``@tk.jit`` kernels too
(``src/thork/kernels/matmul.py:17-71``); its only Blackwell tile matmul is
the single-stage level-06 test kernel (``tests/test_kittens.py:187-274``),
which waits for every TMA load and every MMA in turn.  These kernels use the
same ``tk.kittens`` vocabulary, arranged as a warp-specialised pipeline:

* warp 0 (one lane) is the TMA producer: a ring of ``STAGES`` shared-memory
  stages, each guarded by a ``full`` semaphore (bytes landed) and an
  ``empty`` semaphore (the MMAs reading it have finished);
* warp 1 (one lane) issues the tcgen05 MMAs into a TMEM accumulator; each
  MMA's commit releases its stage;
* warps 2-5 form the epilogue warpgroup: TMEM -> bf16 -> global.

``ncta=1``: one CTA per 128 x 256 output tile, 4 stages of 48 KiB.
``persistent=True``: one CTA per SM looping over 128 x 256 tiles with two
TMEM accumulators, so each tile's epilogue overlaps the next tile's main
loop (``tfull`` / ``tempty`` semaphores; the epilogue warps hand an
accumulator back with ``kittens.arrive``).
``ncta=2``: a cluster pair per 256 x 256 tile (``tcgen05.mma.cta_group::2``):
each CTA loads its 128 rows of A and 128 columns of B into its own shared
memory (each CTA issues its own loads), both CTAs' loads count on the leader's ``full``
semaphore, the leader issues the MMA and its commits land in both CTAs;
6 stages of 32 KiB per CTA.

The stage loop is unrolled at trace time (Python lists of tiles and
semaphores): round r uses stage s for k-block ``r * STAGES + s``, and the
k-blocks past the end of the last round are skipped.  K must be a multiple
of 64, M and N of the tile.  Call as ``k(C, A, B)`` with bf16 (or uint16) arrays
or device arrays.
"""

from .. import dtypes as dt
from .. import kittens as kt
from ..jit import BoundKernel, jit
from ..tracer import if_, local, range as tk_range, syncthreads
from ..types import BlockIdx, GridDim, KittensGlobal, ThreadIdx, Uint

BM, BK = 128, 64


def _shape_check(M, N, K, bm, bn):
    if M % bm or N % bn or K % BK or K <= 0:
        raise ValueError(
            f"tile_matmul: M % {bm}, N % {bn} and K % {BK} must be 0 (K > 0); "
            f"got M={M}, N={N}, K={K}")


def _one_cta(M: int, N: int, K: int, stages: int = 4) -> BoundKernel:
    BN = 256
    _shape_check(M, N, K, BM, BN)
    bf = dt.bfloat16
    G = KittensGlobal
    stage_bytes = (BM * BK + BK * BN) * 2

    @jit
    def tile_matmul_1cta(A: G[bf, (BM, BK)], B: G[bf, (BK, BN)], C: G[bf, (BM, BN)],
                         k_len: Uint, n_len: Uint, bid: Uint[BlockIdx], tid: Uint[ThreadIdx]):
        warp = tid // 32
        lane = tid % 32
        bm = bid // (n_len // BN)
        bn = bid % (n_len // BN)
        a_s = [kt.st_bf(BM, BK) for _ in range(stages)]
        b_s = [kt.st_bf(BK, BN) for _ in range(stages)]
        full = [kt.semaphore() for _ in range(stages)]
        empty = [kt.semaphore() for _ in range(stages)]
        done = kt.semaphore()
        with if_(tid == 0):
            for s in range(stages):
                kt.init_semaphore(full[s], 0, 1)
                kt.init_semaphore(empty[s], 0, 1)
            kt.init_semaphore(done, 0, 1)
        syncthreads()
        alloc = kt.tensor_allocator()
        acc = kt.tt_fl(BM, BN)
        with if_(tid == 0):
            kt.tensor_alloc(acc, alloc, 0)
        syncthreads()
        nkb = k_len // BK
        rounds = (nkb + (stages - 1)) // stages
        with if_(warp == 0):
            with if_(lane == 0):
                ph = local(dt.int32, 0)
                for r in tk_range(rounds):
                    for s in range(stages):
                        kb = r * stages + s
                        with if_(kb < nkb):
                            kt.wait(empty[s], ph ^ 1)
                            kt.tma.expect_bytes(full[s], stage_bytes)
                            kt.tma.load_async(a_s[s], A, (bm, kb), full[s])
                            kt.tma.load_async(b_s[s], B, (kb, bn), full[s])
                    ph ^= 1
        with if_(warp == 1):
            with if_(lane == 0):
                ph = local(dt.int32, 0)
                for r in tk_range(rounds):
                    for s in range(stages):
                        with if_(r * stages + s < nkb):
                            kt.wait(full[s], ph)
                            if s == 0:
                                with if_(r == 0) as first:
                                    kt.warpgroup.mm_AB(acc, a_s[s], b_s[s], empty[s])
                                with first.else_():
                                    kt.warpgroup.mma_AB(acc, a_s[s], b_s[s], empty[s])
                            else:
                                kt.warpgroup.mma_AB(acc, a_s[s], b_s[s], empty[s])
                    ph ^= 1
                kt.tcgen05_commit(done)
        with if_(warp >= 2):
            kt.wait(done, 0)
            kt.warpgroup.store(C, acc, (bm, bn))

    return tile_matmul_1cta.bind(grid=((M // BM) * (N // BN), 1, 1), block=(192, 1, 1))


def _two_cta(M: int, N: int, K: int, stages: int = 6) -> BoundKernel:
    BN = 256          # pair tile columns (MMA N)
    BNH = BN // 2     # B columns held by each CTA
    _shape_check(M, N, K, 2 * BM, BN)
    bf = dt.bfloat16
    G = KittensGlobal
    pair_bytes = 2 * (BM * BK + BK * BNH) * 2  # both CTAs' loads of one stage

    @jit
    def tile_matmul_2cta(A: G[bf, (BM, BK)], B: G[bf, (BK, BNH)], C: G[bf, (BM, BN)],
                         k_len: Uint, n_len: Uint, bid: Uint[BlockIdx], tid: Uint[ThreadIdx]):
        warp = tid // 32
        lane = tid % 32
        rank = kt.cluster_ctarank()
        pair = bid // 2
        bm = pair // (n_len // BN)
        bn = pair % (n_len // BN)
        a_s = [kt.st_bf(BM, BK) for _ in range(stages)]
        b_s = [kt.st_bf(BK, BNH) for _ in range(stages)]
        full = [kt.semaphore() for _ in range(stages)]
        empty = [kt.semaphore() for _ in range(stages)]
        done = kt.semaphore()
        with if_(tid == 0):
            for s in range(stages):
                kt.init_semaphore(full[s], 0, 1)
                kt.init_semaphore(empty[s], 0, 1)
            kt.init_semaphore(done, 0, 1)
        syncthreads()
        alloc = kt.tensor_allocator(ncta=2)  # also the cluster barrier after the inits
        acc = kt.tt_fl(BM, BN)
        with if_(tid == 0):
            kt.tensor_alloc(acc, alloc, 0)
        syncthreads()
        nkb = k_len // BK
        rounds = (nkb + (stages - 1)) // stages
        with if_(warp == 0):
            with if_(lane == 0):
                ph = local(dt.int32, 0)
                for r in tk_range(rounds):
                    for s in range(stages):
                        kb = r * stages + s
                        with if_(kb < nkb):
                            kt.wait(empty[s], ph ^ 1)
                            with if_(rank == 0):
                                kt.tma.pair.expect_bytes(full[s], pair_bytes)
                            kt.tma.pair.load_async(a_s[s], A, (2 * bm + rank, kb), full[s], 0)
                            kt.tma.pair.load_async(b_s[s], B, (kb, 2 * bn + rank), full[s], 0)
                    ph ^= 1
        with if_(warp == 1):
            with if_((lane == 0) & (rank == 0)):
                ph = local(dt.int32, 0)
                for r in tk_range(rounds):
                    for s in range(stages):
                        with if_(r * stages + s < nkb):
                            kt.wait(full[s], ph)
                            if s == 0:
                                with if_(r == 0) as first:
                                    kt.warpgroup.mm2_AB(acc, a_s[s], b_s[s], empty[s])
                                with first.else_():
                                    kt.warpgroup.mma2_AB(acc, a_s[s], b_s[s], empty[s])
                            else:
                                kt.warpgroup.mma2_AB(acc, a_s[s], b_s[s], empty[s])
                    ph ^= 1
                kt.tcgen05_commit(done, ncta=2)
        with if_(warp >= 2):
            kt.wait(done, 0)
            kt.warpgroup.store(C, acc, (2 * bm + rank, bn))

    return tile_matmul_2cta.bind(grid=(2 * (M // (2 * BM)) * (N // BN), 1, 1), block=(192, 1, 1),
                                 cluster=(2, 1, 1))


def _persistent(M: int, N: int, K: int, stages: int = 4, grid: int = None) -> BoundKernel:
    """One CTA per SM looping over 128 x 256 tiles, with two TMEM
    accumulators: the epilogue of one tile overlaps the main loop of the
    next (``tfull`` / ``tempty`` semaphores per accumulator)."""
    BN = 256
    _shape_check(M, N, K, BM, BN)
    if (K // BK) % stages:
        raise ValueError(f"tile_matmul(persistent): K/64 must be a multiple of {stages}, got K={K}")
    bf = dt.bfloat16
    G = KittensGlobal
    stage_bytes = (BM * BK + BK * BN) * 2
    ntiles_host = (M // BM) * (N // BN)

    @jit
    def tile_matmul_persistent(A: G[bf, (BM, BK)], B: G[bf, (BK, BN)], C: G[bf, (BM, BN)],
                               k_len: Uint, n_len: Uint, m_len: Uint, bid: Uint[BlockIdx],
                               nblocks: Uint[GridDim], tid: Uint[ThreadIdx]):
        warp = tid // 32
        lane = tid % 32
        ntn = n_len // BN
        ntiles = (m_len // BM) * ntn
        a_s = [kt.st_bf(BM, BK) for _ in range(stages)]
        b_s = [kt.st_bf(BK, BN) for _ in range(stages)]
        full = [kt.semaphore() for _ in range(stages)]
        empty = [kt.semaphore() for _ in range(stages)]
        tfull = [kt.semaphore() for _ in range(2)]
        tempty = [kt.semaphore() for _ in range(2)]
        with if_(tid == 0):
            for s in range(stages):
                kt.init_semaphore(full[s], 0, 1)
                kt.init_semaphore(empty[s], 0, 1)
            for a in range(2):
                kt.init_semaphore(tfull[a], 0, 1)
                kt.init_semaphore(tempty[a], 4, 0)  # one arrival per epilogue warp
        syncthreads()
        alloc = kt.tensor_allocator()
        acc = [kt.tt_fl(BM, BN) for _ in range(2)]
        with if_(tid == 0):
            kt.tensor_alloc(acc[0], alloc, 0)
            kt.tensor_alloc(acc[1], alloc, BN)
        syncthreads()
        rounds = k_len // (BK * stages)
        with if_(warp == 0):
            with if_(lane == 0):
                ph = local(dt.int32, 0)
                for t in tk_range(bid, ntiles, nblocks):
                    bm = t // ntn
                    bn = t % ntn
                    for r in tk_range(rounds):
                        for s in range(stages):
                            kb = r * stages + s
                            kt.wait(empty[s], ph ^ 1)
                            kt.tma.expect_bytes(full[s], stage_bytes)
                            kt.tma.load_async(a_s[s], A, (bm, kb), full[s])
                            kt.tma.load_async(b_s[s], B, (kb, bn), full[s])
                        ph ^= 1
        with if_(warp == 1):
            with if_(lane == 0):
                ph = local(dt.int32, 0)
                it = local(dt.int32, 0)
                for t in tk_range(bid, ntiles, nblocks):
                    for a in range(2):
                        with if_((it & 1) == a):
                            kt.wait(tempty[a], ((it >> 1) & 1) ^ 1)
                            for r in tk_range(rounds):
                                for s in range(stages):
                                    kt.wait(full[s], ph)
                                    if s == 0:
                                        with if_(r == 0) as first:
                                            kt.warpgroup.mm_AB(acc[a], a_s[s], b_s[s], empty[s])
                                        with first.else_():
                                            kt.warpgroup.mma_AB(acc[a], a_s[s], b_s[s], empty[s])
                                    else:
                                        kt.warpgroup.mma_AB(acc[a], a_s[s], b_s[s], empty[s])
                                ph ^= 1
                            kt.tcgen05_commit(tfull[a])
                    it += 1
        with if_(warp >= 2):
            it = local(dt.int32, 0)
            for t in tk_range(bid, ntiles, nblocks):
                for a in range(2):
                    with if_((it & 1) == a):
                        kt.wait(tfull[a], (it >> 1) & 1)
                        kt.warpgroup.store(C, acc[a], (t // ntn, t % ntn))
                        with if_(lane == 0):
                            kt.arrive(tempty[a])
                it += 1

    if grid is None:
        try:
            from .. import runtime as rt
            grid = rt.sm_count()
        except Exception:  # no device: the B200 SM count
            grid = 148
    return tile_matmul_persistent.bind(grid=(min(grid, ntiles_host), 1, 1), block=(192, 1, 1))


def tile_matmul(M: int, N: int, K: int, ncta: int = 1, stages: int = None,
                persistent: bool = False) -> BoundKernel:
    """Warp-specialised tcgen05 tile matmul written with ``tk.kittens``,
    called as ``k(C, A, B)``.  ``ncta`` selects the 1-CTA (128 x 256 tiles)
    or the cluster-pair (256 x 256 tiles) form; ``stages`` the depth of the
    shared-memory ring (4 and 6 by default)."""
    if persistent:
        if ncta != 1:
            raise ValueError("tile_matmul: the persistent form is 1-CTA")
        return _TileMatmul(_persistent(M, N, K, stages or 4), K, N, M)
    if ncta == 1:
        bound = _one_cta(M, N, K, stages or 4)
    elif ncta == 2:
        bound = _two_cta(M, N, K, stages or 6)
    else:
        raise ValueError(f"tile_matmul: ncta must be 1 or 2, got {ncta}")
    return _TileMatmul(bound, K, N)


class _TileMatmul:
    """``k(C, A, B)``: the bound traced kernel with its K and N arguments
    filled in."""

    __slots__ = ("kernel", "_scalars")

    def __init__(self, kernel: BoundKernel, k: int, n: int, m: int = None):
        self.kernel = kernel
        self._scalars = (int(k), int(n)) + (() if m is None else (int(m),))

    def __call__(self, C, A, B):
        self.kernel(A, B, C, *self._scalars)

    def prepare(self, C, A, B):
        """Device arrays packed once; ``.launch(stream)`` queues the kernel
        without synchronising (``runtime.PreparedLaunch``)."""
        return self.kernel.prepare(A, B, C, *self._scalars)

    @property
    def cuda_source(self) -> str:
        return self.kernel.cuda_source
