"""Multi-GPU execution of the GEMM hot path: one process per GPU, NCCL over
NVLink through libthork_rt.so (no reference counterpart: the reference
hard-codes device 0, ``src/thork/runtime.py:85-105``).

* ``Communicator`` — an NCCL communicator for this rank.  The 128-byte
  unique id is created by rank 0 and exchanged through any key-value store
  with ``set(key, bytes)`` / ``get(key) -> bytes`` (for example a
  ``torch.distributed.TCPStore``); this module itself imports no torch.
* ``row_shard`` / ``col_shard`` — the contiguous partitions used by the
  sharded GEMMs.
* ``sharded_matmul`` — each rank multiplies its contiguous M-row block of A
  by the replicated B and, optionally, all-gathers C so every rank holds
  the full row-major ``M x N`` result (the all-gather is the only
  collective).
* ``sharded_matmul_host`` — the same from host arrays (pinned for full
  PCIe speed): this rank's A rows and B are copied in, C is gathered on the
  devices and this rank's rows are copied back.
* ``FusedGather`` — the same bf16 product with the all-gather fused into
  the GEMM epilogue (P2P stores over NVLink, then a device flag barrier).
* decode shapes split W by contiguous N-column blocks (``col_shard``) with X
  replicated; gathered ``[G, M, N/G]`` blocks become ``M x N`` with
  ``assemble_col_blocks``.
"""

import ctypes
import hashlib
import os
import struct
from typing import Callable, Optional, Tuple

import numpy as np

from . import runtime as rt

DT_BF16 = 4
DT_F32 = 3


def row_shard(m: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous row range [start, stop) of ``rank`` when ``m`` rows are
    split over ``world`` ranks (the first ``m % world`` ranks get one more)."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"rank {rank} out of range for world size {world}")
    base, extra = divmod(m, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def col_shard(n: int, world: int, rank: int, align: int = 8) -> Tuple[int, int]:
    """Contiguous column range of ``rank``; widths are multiples of ``align``
    (16-byte TMA rows) except possibly the last."""
    if n % align:
        raise ValueError(f"N={n} must be a multiple of {align}")
    s, e = row_shard(n // align, world, rank)
    return s * align, e * align


def assemble_col_blocks(gathered: np.ndarray, widths) -> np.ndarray:
    """Turn all-gathered column blocks (concatenated ``[M, w_r]`` row-major
    blocks, rank order) into one ``M x sum(w)`` row-major matrix."""
    widths = list(widths)
    total = sum(widths)
    flat = gathered.reshape(-1)
    m = flat.size // total
    out = np.empty((m, total), gathered.dtype)
    off = col = 0
    for w in widths:
        out[:, col:col + w] = flat[off:off + m * w].reshape(m, w)
        off += m * w
        col += w
    return out


def gather_slot(m_total: int, n: int, world: int, rank: int) -> Tuple[int, int]:
    """(element offset, element count) of ``rank``'s rows inside the
    gathered row-major ``m_total x n`` matrix; the all-gather needs equal
    counts, so rows must split evenly."""
    if m_total % world:
        raise ValueError(f"gather needs M={m_total} divisible by world size {world}")
    start, stop = row_shard(m_total, world, rank)
    return start * n, (stop - start) * n


class Communicator:
    """An NCCL communicator for this process's rank (one GPU per process)."""

    def __init__(self, rank: int, world: int, store=None, key: str = "thork_nccl_id",
                 unique_id: Optional[bytes] = None):
        rt.get_device()
        self.rank, self.world = int(rank), int(world)
        if unique_id is None:
            if store is None:
                raise ValueError("Communicator needs a store or a unique_id")
            if self.rank == 0:
                buf = (ctypes.c_uint8 * 128)()
                rt.check(rt.lib().thork_nccl_get_unique_id(buf), "nccl unique id")
                unique_id = bytes(buf)
                store.set(key, unique_id)
            else:
                unique_id = bytes(store.get(key))
        if len(unique_id) != 128:
            raise ValueError("NCCL unique id must be 128 bytes")
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        h = ctypes.c_void_p()
        rt.check(rt.lib().thork_nccl_comm_init_rank(ctypes.byref(h), self.world, uid, self.rank),
                 "nccl comm init")
        self.handle = h.value

    def allgather(self, send_ptr: int, recv_ptr: int, count: int, dtype: int,
                  stream: Optional[rt.Stream] = None) -> None:
        """recv[r*count:(r+1)*count] = send of rank r (elements of ``dtype``)."""
        rt.check(rt.lib().thork_nccl_allgather(send_ptr, recv_ptr, count, dtype, self.handle,
                                               stream.handle if stream else None), "nccl allgather")

    def allreduce_sum(self, ptr: int, count: int, dtype: int, stream: Optional[rt.Stream] = None):
        rt.check(rt.lib().thork_nccl_allreduce_sum(ptr, count, dtype, self.handle,
                                                   stream.handle if stream else None),
                 "nccl allreduce")

    def close(self) -> None:
        if getattr(self, "handle", None):
            rt.lib().thork_nccl_comm_destroy(self.handle)
            self.handle = None


def serve_fd(name: str, fd: int, payload: bytes, nclients: int, timeout: float = 60.0) -> None:
    """Hand ``fd`` (and ``payload``) to ``nclients`` processes that call
    ``receive_fd(name)``: an abstract-namespace Unix socket, SCM_RIGHTS
    messages.  Returns once every client has been served; raises
    ``TimeoutError`` when one does not connect in time."""
    import socket
    srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    try:
        srv.bind("\0" + name)
        srv.listen(max(nclients, 1))
        srv.settimeout(timeout)
        for _ in range(nclients):
            try:
                conn, _ = srv.accept()
            except socket.timeout as e:
                raise TimeoutError(f"serve_fd({name}): a client did not connect") from e
            with conn:
                socket.send_fds(conn, [payload], [fd])
    finally:
        srv.close()


def receive_fd(name: str, timeout: float = 60.0):
    """The client side of ``serve_fd``: returns (fd, payload); the caller
    owns and closes the received descriptor."""
    import socket
    import time
    t0 = time.monotonic()
    while True:
        cli = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        try:
            cli.connect("\0" + name)
            cli.settimeout(timeout)
            payload, fds, _, _ = socket.recv_fds(cli, 4096, 1)
            if not fds:
                raise RuntimeError(f"receive_fd({name}): no descriptor received")
            return fds[0], payload
        except (ConnectionRefusedError, FileNotFoundError):
            if time.monotonic() - t0 > timeout:
                raise TimeoutError(f"receive_fd({name}): nobody serves it") from None
            time.sleep(0.01)
        finally:
            cli.close()


class MulticastSetupError(RuntimeError):
    """Setting up a multicast buffer failed on some rank; every rank of the
    group raises it together (after releasing what it held)."""


class _Multicast:
    """This rank's part of an NVLink multicast buffer (``thork_mc_*``): one
    object for the group, this GPU's memory bound to it, an ordinary view
    (``local``) and a multicast view (``multi``) where one store reaches
    every GPU.

    Every set-up step ends with ``agree(ok)`` (True only if every rank's
    step succeeded), so all ranks take the same path: when any rank fails,
    every rank releases what it holds and raises, and no rank is left
    waiting in a collective while its memory is bound."""

    def __init__(self, rank: int, world: int, nbytes: int, name: str,
                 agree: Callable[[bool], bool]):
        self.obj = None
        self.local = self.multi = 0
        L = rt.lib()
        err = None
        try:
            if rank == 0:
                obj, fd, size = ctypes.c_void_p(), ctypes.c_int(), ctypes.c_size_t()
                rt.check(L.thork_mc_create(nbytes, world, ctypes.byref(obj), ctypes.byref(fd),
                                           ctypes.byref(size)), "multicast create")
                self.obj, self.bytes = obj.value, size.value
                serve_fd(name, fd.value, struct.pack("<Q", self.bytes), world - 1)
            else:
                fd, payload = receive_fd(name)
                try:
                    self.bytes = struct.unpack("<Q", payload[:8])[0]
                    obj = ctypes.c_void_p()
                    rt.check(L.thork_mc_import(fd, self.bytes, ctypes.byref(obj)),
                             "multicast import")
                    self.obj = obj.value
                finally:
                    os.close(fd)
        except Exception as e:  # noqa: BLE001 - decided together below
            err = e
        self._step(agree, err, "share the multicast object")
        def add():
            # host-side fault injection for tests: this rank fails to add its
            # device, after every rank holds the object and before any binds
            if os.environ.get("THORK_FAULT_MC_SETUP", "") == str(rank):
                raise RuntimeError("injected multicast set-up failure (THORK_FAULT_MC_SETUP)")
            rt.check(L.thork_mc_add_device(self.obj), "multicast add device")
        self._step(agree, self._try(add), "add every device")

        def bind():
            local, multi = ctypes.c_void_p(), ctypes.c_void_p()
            rt.check(L.thork_mc_bind(self.obj, ctypes.byref(local), ctypes.byref(multi)),
                     "multicast bind")
            self.local, self.multi = local.value, multi.value
            rt.check(L.thork_memset(self.local, 0, self.bytes, None), "multicast buffer clear")
            rt.check(L.thork_device_synchronize(), "synchronize")
        # every GPU's memory is bound and clear before any store
        self._step(agree, self._try(bind), "bind every GPU's memory")

    @staticmethod
    def _try(fn):
        try:
            fn()
            return None
        except Exception as e:  # noqa: BLE001 - decided together by the caller
            return e

    def _step(self, agree, err, what: str) -> None:
        if agree(err is None):
            return
        self.release()
        raise MulticastSetupError(f"multicast buffer: could not {what} on every rank"
                                  + (f" (this rank: {err})" if err is not None else ""))

    def release(self) -> None:
        if self.obj:
            obj, self.obj = self.obj, None
            rt.check(rt.lib().thork_mc_release(obj), "multicast release")


def multicast_supported() -> bool:
    """Whether the current GPU can join NVLink multicast buffers."""
    v = ctypes.c_int(0)
    rt.check(rt.lib().thork_mc_supported(ctypes.byref(v)), "multicast supported")
    return bool(v.value)


class _View:
    """A borrowed device pointer in the shape ``DeviceArray`` expects of its
    buffer (no ownership)."""

    __slots__ = ("ptr", "nbytes")

    def __init__(self, ptr: int, nbytes: int):
        self.ptr, self.nbytes = int(ptr), int(nbytes)


class FusedGather:
    """Fused GEMM + all-gather over NVLink peer memory.

    Every rank allocates, in one ``cudaMalloc``, ``slots`` full
    ``m_total x n`` bf16 result buffers and a flag page, exports the
    allocation with CUDA IPC and opens every peer's (the 64-byte handles and
    each GPU's PCI location travel in one NCCL all-gather).  ``matmul`` runs
    this rank's A rows through ``thork_gemm_bf16_allgather``: the GEMM's
    epilogue stores each finished C tile into this GPU's result buffer and,
    with P2P stores over NVLink, into the same rows of every peer's, so the
    transfer overlaps the remaining tiles; a flag barrier kernel
    (``thork_peer_barrier``) then orders every peer's stores before whatever
    this rank queues next.  No NCCL call is on the data path.

    ``mode="multimem"``: the result slots live in an NVLink multicast buffer
    instead (``thork_mc_*``: every GPU's memory bound to one multicast
    object); the epilogue stores each line of this rank's rows once through
    the multicast view and the NVSwitch delivers it to every GPU, so the
    GPU's outgoing NVLink traffic and store count do not grow with the
    number of peers.  Only the flag page is exchanged through CUDA IPC.
    ``mode="auto"`` takes multimem for three or more ranks when every GPU
    supports it, else p2p, and falls back to p2p (on every rank together)
    when setting up the multicast buffer fails.

    Results rotate through the slots: consume a call's result (stream-ordered
    on this rank) before making the next call.  Requires one GPU per rank
    and at most 8 ranks.  ``close()`` is collective; with multimem, call it
    (every rank) before the process exits.
    """

    SLOTS = 2

    def __init__(self, comm: Communicator, m_total: int, n: int, mode: str = "p2p"):
        L = rt.lib()
        self.comm = comm
        self.rank, self.world = comm.rank, comm.world
        if not (1 <= self.world <= 8):
            raise ValueError(f"fused all-gather supports 1..8 ranks, got {self.world}")
        if mode not in ("p2p", "multimem", "auto"):
            raise ValueError(f"unknown fused all-gather mode {mode!r}")
        self.m_total, self.n = int(m_total), int(n)
        self.slot_bytes = ((self.m_total * self.n * 2 + 255) // 256) * 256
        self.mc = None
        if mode == "auto":
            # every rank must take the same decision: agree through NCCL
            flag = rt.DeviceArray((1,), np.float32)
            rt.copy_htod(flag.ptr, np.array([1.0 if multicast_supported() else 0.0], np.float32))
            comm.allreduce_sum(flag.ptr, 1, DT_F32)
            rt.check(L.thork_device_synchronize(), "synchronize")
            # at two ranks both ways measured the same; from three on, one
            # multicast store per line beats a store per peer
            mode = "multimem" if flag.to_host()[0] == self.world and self.world >= 3 else "p2p"
            try:
                self._setup(mode)
            except MulticastSetupError:
                # every rank saw the same failure (agreed): fall back together
                self._setup("p2p")
            return
        self._setup(mode)

    def _setup(self, mode: str) -> None:
        L = rt.lib()
        comm = self.comm
        self.mc = None
        self.mode = mode
        # p2p: the slots and the flag page in one IPC-shared allocation;
        # multimem: only the flag page is shared through IPC
        self.flag_off = self.SLOTS * self.slot_bytes if mode == "p2p" else 0
        self.total_bytes = self.flag_off + 256
        dev = rt.get_device()
        base = ctypes.c_void_p()
        rt.check(L.thork_malloc(self.total_bytes, ctypes.byref(base)), "fused gather buffer")
        self.base = base.value
        rt.check(L.thork_memset(self.base + self.flag_off, 0, 256, None), "flag page clear")
        handle = (ctypes.c_uint8 * 64)()
        rt.check(L.thork_ipc_handle(self.base, handle), "ipc handle")
        loc = np.array([rt.device_attr(a, dev) for a in (7, 8, 9)] + [self.rank], dtype=np.int32)
        mine = bytes(handle) + loc.tobytes()
        rec = len(mine)
        send = rt.DeviceArray((rec,), np.uint8)
        recv = rt.DeviceArray((rec * self.world,), np.uint8)
        rt.copy_htod(send.ptr, np.frombuffer(mine, np.uint8).copy())
        comm.allgather(send.ptr, recv.ptr, rec, 0)
        rt.check(L.thork_device_synchronize(), "synchronize")
        allrec = recv.to_host().reshape(self.world, rec)
        locs = [tuple(allrec[q, 64:].view(np.int32)[:3]) for q in range(self.world)]
        if len(set(locs)) != self.world:
            self._free_own()
            raise RuntimeError("fused all-gather needs one GPU per rank; ranks share a GPU: "
                               f"{locs}")
        self.peer_base = [0] * self.world
        self.peer_base[self.rank] = self.base
        try:
            for q in range(self.world):
                if q == self.rank:
                    continue
                h = (ctypes.c_uint8 * 64).from_buffer_copy(allrec[q, :64].tobytes())
                p = ctypes.c_void_p()
                rt.check(L.thork_ipc_open(h, ctypes.byref(p)), f"ipc open (rank {q})")
                self.peer_base[q] = p.value
        except Exception:
            self._close_peers()
            self._free_own()
            raise
        self.peers = [q for q in range(self.world) if q != self.rank]
        self.epoch = 0
        self.calls = 0
        # completion counts per 128 x 64 unit of C for the push-warp
        # variants (this GPU only)
        rows = max(e - s for s, e in (row_shard(self.m_total, self.world, q)
                                      for q in range(self.world)))
        self.tile_flags = rt.DeviceArray((((rows + 127) // 128) * ((self.n + 63) // 64),),
                                         np.uint32)
        self.tile_flags.zero()
        self.flag_ptrs = (ctypes.c_void_p * 8)(*[b + self.flag_off for b in self.peer_base])
        # every rank has opened every handle (and cleared its flags) before
        # any peer store can arrive
        comm.allgather(send.ptr, recv.ptr, rec, 0)
        rt.check(L.thork_device_synchronize(), "synchronize")
        if mode == "multimem":
            name = "thork-mc-" + hashlib.sha1(allrec[0, :64].tobytes()).hexdigest()[:24]
            try:
                self.mc = _Multicast(self.rank, self.world, self.SLOTS * self.slot_bytes, name,
                                     self._agree)
            except Exception:
                self._close_peers()
                self._free_own()
                raise

    def _agree(self, ok: bool) -> bool:
        """Collective: True when every rank passes ok=True (an NCCL sum,
        waited on); also a host barrier."""
        if getattr(self, "_bar", None) is None:
            self._bar = rt.DeviceArray((1,), np.float32)
        rt.copy_htod(self._bar.ptr, np.array([1.0 if ok else 0.0], np.float32))
        self.comm.allreduce_sum(self._bar.ptr, 1, DT_F32)
        rt.check(rt.lib().thork_device_synchronize(), "synchronize")
        return float(self._bar.to_host()[0]) == float(self.world)

    def _host_barrier(self) -> None:
        self._agree(True)

    def slot_ptr(self, slot: int, rank: Optional[int] = None) -> int:
        if self.mc is not None:
            if rank is not None and rank != self.rank:
                raise ValueError("multimem mode maps no peer result buffers")
            return self.mc.local + (slot % self.SLOTS) * self.slot_bytes
        b = self.base if rank is None else self.peer_base[rank]
        return b + (slot % self.SLOTS) * self.slot_bytes

    def result(self, slot: int) -> "rt.DeviceArray":
        """The full ``m_total x n`` bf16 result held in ``slot`` on this rank."""
        return rt.DeviceArray((self.m_total, self.n), np.uint16,
                              buffer=_View(self.slot_ptr(slot), self.m_total * self.n * 2))

    def barrier(self, stream: Optional[rt.Stream] = None) -> None:
        """Device-side flag barrier over all ranks (stream-ordered)."""
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        rt.check(rt.lib().thork_peer_barrier(self.base + self.flag_off, self.flag_ptrs,
                                             self.world, self.rank, self.epoch,
                                             stream.handle if stream else None), "peer barrier")

    def matmul(self, a_local: "rt.DeviceArray", b: "rt.DeviceArray",
               stream: Optional[rt.Stream] = None, gemm_done: Optional[rt.Event] = None, *,
               dtype: str = "bf16", scale_a: float = 1.0, scale_b: float = 1.0,
               variant: int = 0) -> "rt.DeviceArray":
        """``C = A @ B`` with this rank holding rows ``row_shard(m_total)`` of
        A (bf16, or e4m3 with C scaled by ``scale_a * scale_b``); returns
        (stream-ordered) the full bf16 C on this rank."""
        if dtype not in ("bf16", "e4m3"):
            raise ValueError(f"unknown GEMM dtype {dtype!r}")
        start, stop = row_shard(self.m_total, self.world, self.rank)
        k = a_local.shape[1]
        if a_local.shape[0] != stop - start or tuple(b.shape) != (k, self.n):
            raise ValueError(f"shape mismatch: A rows {a_local.shape}, B {b.shape}, "
                             f"shard {stop - start} x {k}, N {self.n}")
        slot = self.calls % self.SLOTS
        self.calls += 1  # also the epoch of the tile flags
        sh = stream.handle if stream else None
        L = rt.lib()
        if self.mc is not None:
            dst = self.mc.multi + slot * self.slot_bytes
            if dtype == "bf16":
                rc = L.thork_gemm_bf16_allgather_mc(a_local.ptr, b.ptr, dst, stop - start, self.n, k,
                                                    start, sh)
            else:
                rc = L.thork_gemm_e4m3_allgather_mc(a_local.ptr, b.ptr, dst, stop - start, self.n, k,
                                                    start, float(scale_a), float(scale_b), sh)
            rt.check(rc, "fused gemm + multicast all-gather")
            if gemm_done is not None:
                gemm_done.record(stream)
            self.barrier(stream)
            return self.result(slot)
        peers = (ctypes.c_void_p * 7)(*[self.slot_ptr(slot, q) for q in self.peers])
        args = (a_local.ptr, b.ptr, self.slot_ptr(slot), peers, len(self.peers), stop - start,
                self.n, k, start, self.tile_flags.ptr, self.calls & 0xFFFFFFFF)
        if dtype == "bf16":
            rc = L.thork_gemm_bf16_allgather(*args, int(variant), sh)
        else:
            rc = L.thork_gemm_e4m3_allgather(*args, float(scale_a), float(scale_b), int(variant), sh)
        rt.check(rc, "fused gemm + all-gather")
        if gemm_done is not None:
            gemm_done.record(stream)
        self.barrier(stream)
        return self.result(slot)

    def _close_peers(self) -> None:
        for q, p in enumerate(getattr(self, "peer_base", [])):
            if q != self.rank and p:
                rt.lib().thork_ipc_close(p)
                self.peer_base[q] = 0

    def _free_own(self) -> None:
        if getattr(self, "base", 0):
            rt.lib().thork_free(self.base)
            self.base = 0

    def close(self) -> None:
        """Collective: waits until no peer can still store here, then
        releases the mappings and the buffer."""
        if not getattr(self, "base", 0):
            return
        rt.check(rt.lib().thork_device_synchronize(), "synchronize")
        self.barrier(None)
        rt.check(rt.lib().thork_device_synchronize(), "synchronize")
        if self.mc is not None:
            self._host_barrier()  # no rank stores through the multicast view any more
            self.mc.release()
            self.mc = None
        self._close_peers()
        self._free_own()


def _gemm_launcher(dtype: str, m: int, n: int, k: int, scale: float = 1.0,
                   variant: int = 1) -> Callable:
    L = rt.lib()
    # variant 1 (whole 128 x 256 tiles, as in the fused all-gather) whenever C
    # is gathered, so both ways of gathering C produce the same bits; the
    # library's automatic choice (0) when nothing is gathered
    if dtype == "bf16":
        return lambda a, b, c, s: L.thork_gemm_bf16(a, b, c, m, n, k, variant, s)
    if dtype == "e4m3":
        return lambda a, b, c, s: L.thork_gemm_e4m3(a, b, c, m, n, k, float(scale), 1.0, variant, s)
    raise ValueError(f"unknown GEMM dtype {dtype!r}")


def sharded_matmul(comm: Optional[Communicator], a_local: "rt.DeviceArray", b: "rt.DeviceArray",
                   c_out: "rt.DeviceArray", m_total: int, *, dtype: str = "bf16",
                   scale: float = 1.0, gather: bool = True,
                   stream: Optional[rt.Stream] = None, gemm_done: Optional[rt.Event] = None) -> None:
    """This rank's share of ``C = A @ B`` with A split by contiguous rows.

    ``a_local`` holds rows ``row_shard(m_total, world, rank)`` of A; ``b`` is
    the full ``K x N`` matrix.  With ``gather`` the full ``m_total x N`` C is
    all-gathered into ``c_out`` on every rank (rows must split evenly);
    otherwise ``c_out`` receives this rank's rows only.  Queued on ``stream``.
    """
    world = comm.world if comm is not None else 1
    rank = comm.rank if comm is not None else 0
    start, stop = row_shard(m_total, world, rank)
    m_loc = stop - start
    k = a_local.shape[1]
    n = b.shape[1]
    if a_local.shape[0] != m_loc or b.shape[0] != k:
        raise ValueError(f"shape mismatch: A rows {a_local.shape}, B {b.shape}, shard {m_loc}")
    local_only = not gather or world == 1
    launch = _gemm_launcher(dtype, m_loc, n, k, scale, variant=0 if local_only else 1)
    sh = stream.handle if stream else None
    if local_only:
        rt.check(launch(a_local.ptr, b.ptr, c_out.ptr, sh), "sharded gemm")
        if gemm_done is not None:
            gemm_done.record(stream)
        return
    # the local rows land in their final place inside the gathered buffer,
    # and NCCL's in-place all-gather (send == recv + rank*count) fills the rest
    off_elems, count = gather_slot(m_total, n, world, rank)
    rt.check(launch(a_local.ptr, b.ptr, c_out.ptr + 2 * off_elems, sh), "sharded gemm")
    if gemm_done is not None:
        gemm_done.record(stream)
    comm.allgather(c_out.ptr + 2 * off_elems, c_out.ptr, count, DT_BF16, stream)


class _HostStaging:
    """Device buffers (and a side stream) reused across
    ``sharded_matmul_host`` calls."""

    def __init__(self):
        self.bufs = {}
        self._side = None

    def side(self):
        if self._side is None:
            self._side = (rt.Stream(), rt.Event())
        return self._side

    def get(self, key, shape, dtype):
        b = self.bufs.get(key)
        if b is None or b.shape != tuple(shape) or b.dtype != np.dtype(dtype):
            b = rt.empty(shape, dtype)
            self.bufs[key] = b
        return b


_staging = _HostStaging()


def replicate_host_rows(comm: Optional[Communicator], host: np.ndarray, dev: "rt.DeviceArray",
                        stream: rt.Stream) -> int:
    """Put the full row-major ``host`` array into ``dev`` on every rank while
    each rank copies only its contiguous ``1/world`` of the rows over PCIe;
    NCCL's in-place all-gather over NVLink supplies the rest.  Falls back to
    a full copy when the rows do not split evenly.  Returns the bytes this
    rank copied from the host."""
    host = np.ascontiguousarray(host)
    world = comm.world if comm is not None else 1
    rows = host.shape[0]
    if world == 1 or rows % world:
        rt.copy_htod(dev.ptr, host, stream, sync=False)
        return host.nbytes
    start, stop = row_shard(rows, world, comm.rank)
    row_bytes = host.nbytes // rows
    rt.copy_htod(dev.ptr + start * row_bytes, host[start:stop], stream, sync=False)
    count = (stop - start) * row_bytes
    comm.allgather(dev.ptr + start * row_bytes, dev.ptr, count, 0, stream)  # bytes (uint8)
    return count


def sharded_matmul_host(comm: Optional[Communicator], a_rows: np.ndarray, b: np.ndarray,
                        c_rows: np.ndarray, m_total: int, *, dtype: str = "bf16",
                        scale: float = 1.0, fused: Optional[FusedGather] = None) -> None:
    """Host-array form of ``sharded_matmul``: copies this rank's A rows and
    its share of B's rows to the device (B is completed over NVLink by
    ``replicate_host_rows``), computes and all-gathers C on the devices
    (through ``fused`` when given, else NCCL), and copies this rank's rows of
    C back into ``c_rows``.  Synchronous."""
    stream = rt._dispatch_stream()
    a_dev = _staging.get("a", a_rows.shape, a_rows.dtype)
    b_dev = _staging.get("b", b.shape, b.dtype)
    world = comm.world if comm is not None else 1
    if fused is not None and world > 1:
        # B's NVLink all-gather runs on a side stream while A's rows cross PCIe
        side, ev = _staging.side()
        replicate_host_rows(comm, b, b_dev, side)
        ev.record(side)
        rt.copy_htod(a_dev.ptr, np.ascontiguousarray(a_rows), stream, sync=False)
        stream.wait(ev)
        c = fused.matmul(a_dev, b_dev, stream, dtype=dtype, scale_a=scale)
        start, _ = row_shard(m_total, world, comm.rank)
        rt.copy_dtoh(c_rows, c.ptr + start * b.shape[1] * 2, stream, sync=False)
        stream.synchronize()
        return
    rows_out = m_total if world > 1 else a_rows.shape[0]
    c_dev = _staging.get("c", (rows_out, b.shape[1]), np.uint16)
    replicate_host_rows(comm, b, b_dev, stream)
    rt.copy_htod(a_dev.ptr, np.ascontiguousarray(a_rows), stream, sync=False)
    sharded_matmul(comm, a_dev, b_dev, c_dev, m_total, dtype=dtype, scale=scale,
                   gather=world > 1, stream=stream)
    rank = comm.rank if comm is not None else 0
    start, _ = row_shard(m_total, world, rank)
    off = (start * b.shape[1] * 2) if world > 1 else 0
    rt.copy_dtoh(c_rows, c_dev.ptr + off, stream, sync=False)
    stream.synchronize()
