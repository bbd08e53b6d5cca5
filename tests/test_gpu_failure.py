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
