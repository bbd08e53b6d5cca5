"""Failure detection on the GPU without a fault: a traced tile kernel waits
on a semaphore that nothing arrives on.  The bounded wait gives up after
about a second, the kernel records a status and returns, the host raises,
and the context stays usable for the next launch."""

import time

import numpy as np
import pytest

import thork_b200 as tk
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_context_survives():
    G = tk.kittens.Global

    @tk.jit
    def never_signalled(A: G[tk.dt.bfloat16], tid: tk.Uint[tk.ThreadIdx]):
        sem = tk.kittens.semaphore()
        with tk.if_(tid == 0):
            tk.kittens.init_semaphore(sem, 1, 0)
        tk.syncthreads()
        tk.kittens.wait(sem, 0)  # nothing arrives: phase 0 never completes

    a = np.zeros((8, 8), np.uint16)
    t0 = time.time()
    with pytest.raises(tk.runtime.CudaError) as ei:
        never_signalled[(1, 1, 1), (32, 1, 1)](a)
    elapsed = time.time() - t0
    assert ei.value.code == tk.runtime.ERR_KERNEL
    assert "bounded wait expired" in str(ei.value)
    assert 0.5 < elapsed < 30.0
    assert tk.runtime.kernel_status() == 0  # the status word was cleared

    # the context is still usable
    x, y = oracle.add_inputs((4096,), seed=1)
    out = np.zeros_like(x)
    tk.kernels.matrix_add((4096,))(out, x, y)
    np.testing.assert_array_equal(out, oracle.add_ref(x, y))


def test_peer_barrier_that_no_peer_joins_times_out_with_a_status():
    """The fused all-gather's flag barrier on one GPU, with a 'peer' flag
    page that nothing writes: the bounded wait expires, the status word
    records the barrier site (20), and the context stays usable."""
    import ctypes
    rt = tk.runtime
    L = rt.lib()
    flags = rt.empty((8,), np.uint32)      # this rank's flags: nobody arrives
    peer = rt.empty((8,), np.uint32)       # stands in for rank 1's page
    flags.zero()
    peer.zero()
    ptrs = (ctypes.c_void_p * 8)(0, peer.ptr)
    rt.kernel_status(clear=True)
    t0 = time.time()
    rt.check(L.thork_peer_barrier(flags.ptr, ptrs, 2, 0, 1, None))
    rt.synchronize()
    elapsed = time.time() - t0
    st = rt.kernel_status(clear=True)
    assert st == (1 | (20 << 8)), hex(st)
    assert 0.5 < elapsed < 30.0
    assert peer.to_host()[0] == 1  # this rank's arrival reached the peer page
    x, y = oracle.add_inputs((4096,), seed=2)
    out = np.zeros_like(x)
    tk.kernels.matrix_add((4096,))(out, x, y)
    np.testing.assert_array_equal(out, oracle.add_ref(x, y))
