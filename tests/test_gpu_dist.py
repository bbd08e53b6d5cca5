"""Multi-GPU parity (skipped with fewer than 2 GPUs): one process per GPU,
A split by contiguous rows, B replicated, the tcgen05 GEMM writes each rank's
rows in place and NCCL all-gathers C; every rank checks the full result
against the oracle.  Also the column-split decode GEMM and its assembly."""

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import datetime
    import torch.distributed as td
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    td.init_process_group("gloo", rank=rank, world_size=world,
                          timeout=datetime.timedelta(seconds=60))
    comm = None
    try:
        import thork_b200 as tk
        from thork_b200 import dist
        from oracle import oracle
        rt = tk.runtime
        rt.set_device(rank)
        uid = [None]
        if rank == 0:
            import ctypes
            buf = (ctypes.c_uint8 * 128)()
            rt.check(rt.lib().thork_nccl_get_unique_id(buf))
            uid = [bytes(buf)]
        td.broadcast_object_list(uid, src=0)
        comm = dist.Communicator(rank, world, unique_id=uid[0])
        m, n, k = 1024, 768, 512
        a, b = oracle.gemm_inputs(m, n, k, seed=3)
        a16, b16 = oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(b)
        s, e = dist.row_shard(m, world, rank)
        A = rt.to_device(np.ascontiguousarray(a16[s:e]))
        B = rt.to_device(b16)
        C = rt.empty((m, n), np.uint16)
        stream = rt.Stream()
        dist.sharded_matmul(comm, A, B, C, m, dtype="bf16", stream=stream)
        stream.synchronize()
        c = oracle.bf16_bits_to_f32(C.to_host())
        err = oracle.max_rel_err(c, oracle.gemm_bf16_ref(a16, b16))
        assert err <= 1e-2, f"rank {rank}: max rel err {err}"
        # host-array form
        c_rows = np.zeros((e - s, n), np.uint16)
        dist.sharded_matmul_host(comm, np.ascontiguousarray(a16[s:e]), b16, c_rows, m)
        np.testing.assert_array_equal(c_rows, C.to_host()[s:e])
        q.put((rank, "ok"))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, repr(exc)))
    finally:
        if comm is not None:
            comm.close()
        td.destroy_process_group()


def test_two_gpu_sharded_gemm_with_nccl_allgather():
    import thork_b200 as tk
    if tk.runtime.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = dict(q.get(timeout=10) for _ in range(2))
    assert results == {0: "ok", 1: "ok"}, results
