"""Multi-GPU host logic on CPU: partitions, gather slots and the column-block
assembly of thork_b200.dist, exercised by world-size-2 gloo processes that
stand in for GPUs (NumPy computes each rank's block)."""

import os
import socket

import numpy as np
import pytest

from thork_b200 import dist


def test_row_shard_partitions_contiguously():
    for m in (1, 7, 8192, 1000):
        for world in (1, 2, 3, 4, 8):
            spans = [dist.row_shard(m, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == m
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        dist.row_shard(8, 2, 2)


def test_col_shard_keeps_16_byte_columns():
    for world in (1, 2, 4, 8):
        spans = [dist.col_shard(14336, world, r) for r in range(world)]
        assert spans[-1][1] == 14336
        assert all(s % 8 == 0 and e % 8 == 0 for s, e in spans)
    with pytest.raises(ValueError):
        dist.col_shard(100, 2, 0)


def test_assemble_col_blocks():
    rng = np.random.default_rng(0)
    y = rng.standard_normal((5, 48)).astype(np.float32)
    widths = [16, 16, 8, 8]
    blocks, c = [], 0
    for w in widths:
        blocks.append(np.ascontiguousarray(y[:, c:c + w]).reshape(-1))
        c += w
    np.testing.assert_array_equal(dist.assemble_col_blocks(np.concatenate(blocks), widths), y)


def test_gather_slot_requires_even_split():
    assert dist.gather_slot(8192, 8192, 8, 3) == (3 * 1024 * 8192, 1024 * 8192)
    with pytest.raises(ValueError):
        dist.gather_slot(10, 4, 4, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as td
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    td.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = n = 64
        k = 32
        rng = np.random.default_rng(0)  # every rank draws the same inputs
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        s, e = dist.row_shard(m, world, rank)
        full = np.zeros(m * n, np.float32)
        off, count = dist.gather_slot(m, n, world, rank)
        full[off:off + count] = (a[s:e] @ b).reshape(-1)  # this rank's GEMM, in place
        parts = [torch.zeros(count) for _ in range(world)]
        td.all_gather(parts, torch.from_numpy(full[off:off + count].copy()))
        gathered = torch.cat(parts).numpy().reshape(m, n)
        np.testing.assert_allclose(gathered, a @ b, rtol=1e-5, atol=1e-5)
        # decode layout: column blocks of W, gathered [G, M, N/G] -> M x N
        x = rng.standard_normal((3, k)).astype(np.float32)
        w = rng.standard_normal((k, 48)).astype(np.float32)
        spans = [dist.col_shard(48, world, r) for r in range(world)]
        c0, c1 = spans[rank]
        mine = torch.from_numpy(np.ascontiguousarray(x @ w[:, c0:c1]).reshape(-1))
        sizes = [3 * (e_ - s_) for s_, e_ in spans]
        outs = [torch.zeros(sz) for sz in sizes]
        td.all_gather(outs, mine)
        y = dist.assemble_col_blocks(torch.cat(outs).numpy(), [e_ - s_ for s_, e_ in spans])
        np.testing.assert_allclose(y, x @ w, rtol=1e-5, atol=1e-5)
        q.put((rank, "ok"))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, repr(exc)))
    finally:
        td.destroy_process_group()


def test_two_rank_gloo_shard_and_gather():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert results == {0: "ok", 1: "ok"}


class _HostComm:
    """An in-place all-gather over host memory for ranks run as threads."""

    def __init__(self, rank, world, shared):
        self.rank, self.world, self.shared = rank, world, shared

    def allgather(self, send_ptr, recv_ptr, count, dtype, stream=None):
        import ctypes
        self.shared["send"][self.rank] = send_ptr
        self.shared["barrier"].wait()
        for r in range(self.world):
            if r != self.rank:
                ctypes.memmove(recv_ptr + r * count, self.shared["send"][r], count)
        self.shared["barrier"].wait()


@pytest.mark.parametrize("rows,world", [(64, 4), (62, 4), (8, 1)])
def test_replicate_host_rows_copies_one_share_per_rank(monkeypatch, rows, world):
    """Each rank copies only its contiguous share of the rows and the
    in-place all-gather completes the array on every rank; rows that do not
    split evenly fall back to a full copy."""
    import ctypes
    import threading
    from types import SimpleNamespace
    copied = []  # bytes of every host copy (list.append is atomic)

    def fake_htod(ptr, arr, stream=None, sync=True):
        arr = np.ascontiguousarray(arr)
        ctypes.memmove(ptr, arr.ctypes.data, arr.nbytes)
        copied.append(arr.nbytes)

    monkeypatch.setattr(dist.rt, "copy_htod", fake_htod)
    host = np.random.default_rng(1).integers(0, 65535, (rows, 24), dtype=np.uint16)
    devs = [np.zeros_like(host) for _ in range(world)]
    shared = {"send": {}, "barrier": threading.Barrier(world)}
    results, errors = [None] * world, []

    def run(r):
        try:
            comm = _HostComm(r, world, shared) if world > 1 else None
            dev = SimpleNamespace(ptr=devs[r].ctypes.data)
            results[r] = dist.replicate_host_rows(comm, host, dev, None)
        except Exception as exc:  # noqa: BLE001 - reported below
            errors.append(exc)
            shared["barrier"].abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=30)
    assert not errors, errors
    for d in devs:
        np.testing.assert_array_equal(d, host)
    share = host.nbytes // world if rows % world == 0 else host.nbytes
    assert results == [share] * world
    assert copied == [share] * world  # one copy per rank, of its share


def _receive_and_write(name, q):
    import os
    from thork_b200 import dist
    fd, payload = dist.receive_fd(name, timeout=30)
    os.write(fd, b"from-child:" + payload)
    os.close(fd)
    q.put("ok")


def test_descriptor_handoff_between_processes():
    """serve_fd / receive_fd hand a file descriptor (and a payload) to other
    processes over an abstract Unix socket, as the multicast buffer setup
    does with the multicast object's descriptor."""
    import multiprocessing as mp
    import os
    import uuid
    from thork_b200 import dist
    r, w = os.pipe()
    name = "thork-test-" + uuid.uuid4().hex[:12]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_receive_and_write, args=(name, q)) for _ in range(2)]
    for p in procs:
        p.start()
    dist.serve_fd(name, w, b"xy", 2, timeout=60)
    os.close(w)
    for p in procs:
        p.join(timeout=60)
    assert [q.get(timeout=10) for _ in procs] == ["ok", "ok"]
    data = b""
    while True:
        chunk = os.read(r, 100)
        if not chunk:
            break
        data += chunk
    os.close(r)
    assert data == b"from-child:xy" * 2


def test_receive_fd_times_out_without_server():
    import uuid
    from thork_b200 import dist
    with pytest.raises(TimeoutError):
        dist.receive_fd("thork-absent-" + uuid.uuid4().hex[:12], timeout=0.2)
