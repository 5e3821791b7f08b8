"""The device status word (needs a B200).

Kernels record a code there only when one of their bounded waits expires.
After ordinary work -- the decode GEMVs and the prefill GEMM on every dtype --
the word must read CLQ_OK.  A wait that runs out must surface as
CLQ_ERR_TIMEOUT through clq_device_status, leave the context usable and clear
on read (the error contract behind local/backend.lisp:148-157, where any
failure of a step becomes an error the caller sees).
"""
import ctypes

import numpy as np
import pytest

from helpers import element_bound_ok

pytestmark = pytest.mark.gpu


def status(clq):
    s = ctypes.c_int(-1)
    assert clq._lib.lib.clq_device_status(ctypes.byref(s)) == 0, clq._lib.last_error()
    return s.value


@pytest.mark.parametrize("dtype", ["q4_k", "q6_k", "q4_0", "q8_0"])
def test_status_stays_clear_through_gemv_and_gemm(cuda, clq, synth, dtype):
    torch = cuda
    assert status(clq) == 0
    n, k = 1000, 2048
    store = clq.Store(dtype, n, k, synth.packed_blocks(dtype, n, k, seed=3))
    for m in (1, 3, 8, 96):
        x = torch.from_numpy(synth.activations(m, k, seed=m)).cuda().to(torch.bfloat16)
        y = store.linear(x)
        assert torch.isfinite(y).all()
    assert status(clq) == 0
    store.close()


def test_an_expired_wait_reports_timeout(cuda, clq, synth, oracle, monkeypatch):
    """A two-rank all-reduce group whose second rank never runs: both receive
    buffers live on this GPU, the launch writes its words into both, then waits
    for the absent rank's words, which nothing writes.  The wait is bounded
    (CLQ_TP_WAIT_POLLS, a test-only knob read when the group is created), so
    the kernel gives up, records CLQ_ERR_TIMEOUT and returns; one kernel waits
    here, for memory no other launch touches.  The status reads the timeout
    once, then clears, and the next product is correct."""
    torch = cuda
    lib = clq._lib.lib
    assert status(clq) == 0
    monkeypatch.setenv("CLQ_TP_WAIT_POLLS", "20000")
    world, cap = 2, 4096
    bufs = []
    for _ in range(world):
        recv, flags = ctypes.c_void_p(), ctypes.c_void_p()
        clq._lib.check(lib.clq_tp_buffers(world, cap, ctypes.byref(recv), ctypes.byref(flags)))
        bufs.append((recv, flags))
    handle = ctypes.c_void_p()
    try:
        R = (ctypes.c_void_p * world)(*[b[0].value for b in bufs])
        F = (ctypes.c_void_p * world)(*[b[1].value for b in bufs])
        clq._lib.check(lib.clq_tp_create(0, world, cap, R, F, ctypes.byref(handle)))
        n, k = 512, 1024
        data = synth.packed_blocks("q4_k", n, k, seed=77)
        store = clq.Store("q4_k", n, k, data)
        x_np = synth.activations(1, k, seed=78)
        x = torch.from_numpy(x_np).cuda()
        out = torch.empty(1, n, device="cuda")
        rc = lib.clq_linear_allreduce_device(store.handle, 0, n, x.data_ptr(), clq._lib.CLQ_X_F32, 1,
                                             out.data_ptr(), n, handle, None)
        assert rc == 0, clq._lib.last_error()
        torch.cuda.synchronize()  # the launch ends by itself: its wait is bounded
        assert clq._lib.STATUS_NAMES[status(clq)] == "CLQ_ERR_TIMEOUT"
        assert status(clq) == 0  # read once, then cleared
        # the context is healthy: an ordinary product matches the oracle
        y = store.linear(x).cpu().numpy()
        ref, mag = oracle.matmul_f64("q4_k", x_np, data, n)
        assert element_bound_ok(y, ref, mag)
        assert status(clq) == 0
        store.close()
    finally:
        torch.cuda.synchronize()
        if handle.value:
            lib.clq_tp_free(handle)
        for recv, flags in bufs:
            lib.clq_tp_buffers_free(recv, flags)
