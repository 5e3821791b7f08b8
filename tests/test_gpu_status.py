"""The device status word after ordinary work (needs a B200).

Kernels record a code there only when one of their bounded pipeline waits
expires; the decode GEMV (bulk-copy pipeline) and the prefill GEMM run here on
every dtype, and the word must read CLQ_OK afterwards.
"""
import ctypes

import pytest

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
