"""Fused GEMM + all-gather over NVLink peer memory (skipped with fewer than
2 GPUs): one process per GPU, each rank's GEMM epilogue stores its C rows
into every rank's result buffer, a device flag barrier closes each call.
Every rank checks the full C of several successive calls (the result slots
rotate) against the oracle and bit-for-bit against the NCCL all-gather
path, on even and uneven row splits."""

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
    comm = fg = None
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
        stream = rt.Stream()
        for m, n, k in ((1024, 768, 512), (1001, 520, 264)):
            fg = dist.FusedGather(comm, m, n)
            b = None
            for call in range(4):
                a, b0 = oracle.gemm_inputs(m, n, k, seed=10 + call)
                if b is None:
                    b = oracle.f32_to_bf16_bits(b0)
                    B = rt.to_device(b)
                a16 = oracle.f32_to_bf16_bits(a)
                s, e = dist.row_shard(m, world, rank)
                A = rt.to_device(np.ascontiguousarray(a16[s:e]))
                variant = 1 + call % 2
                C = fg.matmul(A, B, stream, variant=variant)
                got = C.to_host(stream=stream)  # consumed before the next call
                err = oracle.max_rel_err(oracle.bf16_bits_to_f32(got), oracle.gemm_bf16_ref(a16, b))
                assert err <= 1e-2, f"rank {rank} call {call} {m}x{n}x{k}: max rel err {err}"
                if m % world == 0:
                    ref = rt.empty((m, n), np.uint16)
                    dist.sharded_matmul(comm, A, B, ref, m, dtype="bf16", stream=stream)
                    np.testing.assert_array_equal(got, ref.to_host(stream=stream))
            # host-array form through the same fused path
            c_rows = np.zeros((e - s, n), np.uint16)
            dist.sharded_matmul_host(comm, np.ascontiguousarray(a16[s:e]), b, c_rows, m, fused=fg)
            np.testing.assert_array_equal(c_rows, got[s:e])
            st = rt.kernel_status(clear=True)
            assert st == 0, f"rank {rank}: kernel status {st:#x}"
            fg.close()
            fg = None
        # FP8 e4m3 through the same fused epilogue
        m, n, k = 1024, 512, 256
        fg = dist.FusedGather(comm, m, n)
        a, b = oracle.gemm_inputs(m, n, k, seed=21)
        qa, sa = oracle.quantize_e4m3(a)
        qb, sb = oracle.quantize_e4m3(b)
        s, e = dist.row_shard(m, world, rank)
        C = fg.matmul(rt.to_device(np.ascontiguousarray(qa[s:e])), rt.to_device(qb), stream,
                      dtype="e4m3", scale_a=sa, scale_b=sb)
        got = oracle.bf16_bits_to_f32(C.to_host(stream=stream))
        err = oracle.max_rel_err(got, oracle.gemm_e4m3_ref(qa, sa, qb, sb))
        assert err <= 1e-2, f"rank {rank} e4m3: max rel err {err}"
        fg.close()
        fg = None
        q.put((rank, "ok"))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, repr(exc)))
    finally:
        if fg is not None:
            fg.close()
        if comm is not None:
            comm.close()
        td.destroy_process_group()


@pytest.mark.parametrize("dtype", ["bf16", "e4m3"])
def test_fused_epilogue_on_one_gpu_writes_every_destination(dtype):
    """The peer-store epilogue with 3 destination buffers on the same GPU:
    the rows [row0, row0 + rows) of each must equal the plain GEMM's output,
    bit for bit, and every other row must stay untouched."""
    import ctypes
    import thork_b200 as tk
    from oracle import oracle
    rt = tk.runtime
    L = rt.lib()
    m_total, rows, row0, n, k = 700, 301, 257, 400, 320
    a, b = oracle.gemm_inputs(rows, n, k, seed=5)
    if dtype == "bf16":
        qa, qb = oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(b)
        sa = sb = 1.0
        ref = oracle.gemm_bf16_ref(qa, qb)
    else:
        qa, sa = oracle.quantize_e4m3(a)
        qb, sb = oracle.quantize_e4m3(b)
        ref = oracle.gemm_e4m3_ref(qa, sa, qb, sb)
    A, B = rt.to_device(qa), rt.to_device(qb)
    dests = [rt.to_device(np.full((m_total, n), 0x7E7E, np.uint16)) for _ in range(3)]
    plain = rt.empty((rows, n), np.uint16)
    peers = (ctypes.c_void_p * 7)(dests[1].ptr, dests[2].ptr)
    flags = rt.empty((((rows + 127) // 128) * ((n + 63) // 64),), np.uint32)
    flags.zero()
    if dtype == "bf16":
        rt.check(L.thork_gemm_bf16(A.ptr, B.ptr, plain.ptr, rows, n, k, 1, None))
    else:
        rt.check(L.thork_gemm_e4m3(A.ptr, B.ptr, plain.ptr, rows, n, k, sa, sb, 1, None))
    want = plain.to_host()
    assert oracle.max_rel_err(oracle.bf16_bits_to_f32(want), ref) <= 1e-2
    # both all-gather variants in turn on the same tile flags
    for epoch, variant in enumerate((1, 2, 2, 1, 2), start=1):
        for d in dests:
            rt.check(L.thork_memset(d.ptr, 0x7E, d.nbytes, None))
        if dtype == "bf16":
            rt.check(L.thork_gemm_bf16_allgather(A.ptr, B.ptr, dests[0].ptr, peers, 2, rows, n, k,
                                                 row0, flags.ptr, epoch, variant, None))
        else:
            rt.check(L.thork_gemm_e4m3_allgather(A.ptr, B.ptr, dests[0].ptr, peers, 2, rows, n, k,
                                                 row0, flags.ptr, epoch, sa, sb, variant, None))
        rt.synchronize()
        assert rt.kernel_status() == 0, (epoch, variant)
        first = dests[0].to_host()[row0:row0 + rows]
        np.testing.assert_array_equal(first, want)  # same 128 x 256 tiles as the plain kernel
        for d in dests:
            got = d.to_host()
            np.testing.assert_array_equal(got[row0:row0 + rows], first)
            assert (got[:row0] == 0x7E7E).all() and (got[row0 + rows:] == 0x7E7E).all()


def test_fused_gemm_allgather_over_peer_memory():
    import thork_b200 as tk
    ndev = tk.runtime.device_count()
    if ndev < 2:
        pytest.skip("needs 2 GPUs")
    world = min(ndev, 8)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = dict(q.get(timeout=10) for _ in range(world))
    assert results == {r: "ok" for r in range(world)}, results


def _rank_multimem(rank, world, port, q):
    """The multimem mode: one store per line through an NVLink multicast
    view.  Every rank runs the same collective steps whatever its checks
    find (failures are collected, not raised, until the buffer is released),
    so no rank leaves while its memory is bound to the multicast object."""
    import datetime
    import torch.distributed as td
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    td.init_process_group("gloo", rank=rank, world_size=world,
                          timeout=datetime.timedelta(seconds=60))
    comm = None
    problems = []
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
        stream = rt.Stream()
        for m, n, k in ((1024, 768, 512), (1001, 520, 264)):
            fg = dist.FusedGather(comm, m, n, mode="multimem")
            try:
                assert fg.mode == "multimem"
                b = None
                for call in range(4):
                    a, b0 = oracle.gemm_inputs(m, n, k, seed=30 + call)
                    if b is None:
                        b = oracle.f32_to_bf16_bits(b0)
                        B = rt.to_device(b)
                    a16 = oracle.f32_to_bf16_bits(a)
                    s, e = dist.row_shard(m, world, rank)
                    A = rt.to_device(np.ascontiguousarray(a16[s:e]))
                    got = fg.matmul(A, B, stream).to_host(stream=stream)
                    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(got), oracle.gemm_bf16_ref(a16, b))
                    if err > 1e-2:
                        problems.append(f"{m}x{n}x{k} call {call}: max rel err {err}")
                    if m % world == 0:
                        ref = rt.empty((m, n), np.uint16)
                        dist.sharded_matmul(comm, A, B, ref, m, dtype="bf16", stream=stream)
                        if not np.array_equal(got, ref.to_host(stream=stream)):
                            problems.append(f"{m}x{n}x{k} call {call}: differs from NCCL path")
                if m == 1024:
                    qa, sa = oracle.quantize_e4m3(a)
                    qb, sb = oracle.quantize_e4m3(b0)
                    s, e = dist.row_shard(m, world, rank)
                    got = fg.matmul(rt.to_device(np.ascontiguousarray(qa[s:e])), rt.to_device(qb),
                                    stream, dtype="e4m3", scale_a=sa, scale_b=sb).to_host(stream=stream)
                    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(got),
                                             oracle.gemm_e4m3_ref(qa, sa, qb, sb))
                    if err > 1e-2:
                        problems.append(f"e4m3: max rel err {err}")
                st = rt.kernel_status(clear=True)
                if st:
                    problems.append(f"kernel status {st:#x}")
            finally:
                fg.close()
        q.put((rank, "ok" if not problems else "; ".join(problems)))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, repr(exc)))
    finally:
        if comm is not None:
            comm.close()
        td.destroy_process_group()


def test_fused_gemm_allgather_through_multicast():
    import thork_b200 as tk
    from thork_b200 import dist
    ndev = tk.runtime.device_count()
    if ndev < 2:
        pytest.skip("needs 2 GPUs")
    tk.runtime.set_device(0)
    if not dist.multicast_supported():
        pytest.skip("NVLink multicast not supported here")
    world = min(ndev, 8)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_multimem, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = dict(q.get(timeout=10) for _ in range(world))
    assert results == {r: "ok" for r in range(world)}, results


def _rank_auto_fallback(rank, world, port, q):
    """mode="auto" with an injected multicast set-up failure on rank 1: every
    rank falls back to P2P stores together and the results stay right."""
    import datetime
    import torch.distributed as td
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), THORK_FAULT_MC_SETUP="1")
    td.init_process_group("gloo", rank=rank, world_size=world,
                          timeout=datetime.timedelta(seconds=60))
    comm = fg = None
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
        m, n, k = 1024, 512, 256
        fg = dist.FusedGather(comm, m, n, mode="auto")
        a, b = oracle.gemm_inputs(m, n, k, seed=51)
        a16, b16 = oracle.f32_to_bf16_bits(a), oracle.f32_to_bf16_bits(b)
        s, e = dist.row_shard(m, world, rank)
        stream = rt.Stream()
        got = fg.matmul(rt.to_device(np.ascontiguousarray(a16[s:e])), rt.to_device(b16),
                        stream).to_host(stream=stream)
        err = oracle.max_rel_err(oracle.bf16_bits_to_f32(got), oracle.gemm_bf16_ref(a16, b16))
        mode = fg.mode
        fg.close()
        fg = None
        q.put((rank, "ok" if mode == "p2p" and err <= 1e-2 else f"mode {mode} err {err}"))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, repr(exc)))
    finally:
        if fg is not None:
            fg.close()
        if comm is not None:
            comm.close()
        td.destroy_process_group()


def test_auto_mode_falls_back_to_p2p_together():
    import thork_b200 as tk
    from thork_b200 import dist
    ndev = tk.runtime.device_count()
    if ndev < 3:
        pytest.skip("needs 3 GPUs (auto takes multicast from three ranks)")
    tk.runtime.set_device(0)
    if not dist.multicast_supported():
        pytest.skip("NVLink multicast not supported here")
    world = min(ndev, 8)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_auto_fallback, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = dict(q.get(timeout=10) for _ in range(world))
    assert results == {r: "ok" for r in range(world)}, results
