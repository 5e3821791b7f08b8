"""The host-buffer drop-in call path on the device (needs a B200).

`clq_q4_k_matmul` & co. copy x through mapped page-locked staging with a copy
kernel, remember each thread's weight lookups and replay decode-sized calls
(M <= 8) as CUDA graphs.  These tests drive that state: repeated and
interleaved calls give the first call's bits, a call large enough to move the
staging buffers leaves later calls correct, and `clq_forget` followed by new
bytes at the same host address is seen (the reference's copy-once rule holds
only until the weight is forgotten, `local/weights.lisp:84-89`).
"""
import numpy as np
import pytest

from helpers import element_bound_ok

pytestmark = pytest.mark.gpu


def call(lib, fn, data, x, n, k):
    m = x.shape[0]
    out = np.empty((m, n), np.float32)
    rc = fn(out.ctypes.data, x.ctypes.data, data.ctypes.data, m, n, k)
    assert rc == 0
    return out


def test_repeated_and_interleaved_calls_keep_their_bits(cuda, clq, synth, oracle):
    lib = clq._lib.lib
    lib.clq_clear_cache()
    k = 2048
    a = synth.packed_blocks("q4_k", 512, k, seed=11)
    b = synth.packed_blocks("q6_k", 300, k, seed=12)
    xs = {m: synth.activations(m, k, seed=20 + m) for m in (1, 3, 8)}
    first = {}
    for m, x in xs.items():
        first[("a", m)] = call(lib, lib.clq_q4_k_matmul, a, x, 512, k)
        first[("b", m)] = call(lib, lib.clq_q6_k_matmul, b, x, 300, k)
        for name, data, n, dt in (("a", a, 512, "q4_k"), ("b", b, 300, "q6_k")):
            ref, mag = oracle.matmul_f64(dt, x, data, n)
            assert element_bound_ok(first[(name, m)], ref, mag), (name, m)
    for _ in range(3):  # graph replays, in a different order
        for m in (8, 1, 3):
            got_b = call(lib, lib.clq_q6_k_matmul, b, xs[m], 300, k)
            got_a = call(lib, lib.clq_q4_k_matmul, a, xs[m], 512, k)
            assert np.array_equal(got_a.view(np.uint32), first[("a", m)].view(np.uint32))
            assert np.array_equal(got_b.view(np.uint32), first[("b", m)].view(np.uint32))
    lib.clq_clear_cache()


def test_calls_after_the_staging_buffers_move(cuda, clq, synth, oracle):
    lib = clq._lib.lib
    lib.clq_clear_cache()
    n, k = 256, 4096
    data = synth.packed_blocks("q4_k", n, k, seed=13)
    x1 = synth.activations(1, k, seed=31)
    before = call(lib, lib.clq_q4_k_matmul, data, x1, n, k)
    before2 = call(lib, lib.clq_q4_k_matmul, data, x1, n, k)
    assert np.array_equal(before.view(np.uint32), before2.view(np.uint32))
    # a decode-sized call with a wider weight grows the output staging
    wide = synth.packed_blocks("q4_k", 4096, k, seed=14)
    x8 = synth.activations(8, k, seed=32)
    got = call(lib, lib.clq_q4_k_matmul, wide, x8, 4096, k)
    ref, mag = oracle.matmul_f64("q4_k", x8, wide[: 64 * (k // 256) * 144], 64)
    assert element_bound_ok(got[:, :64], ref, mag)
    after = call(lib, lib.clq_q4_k_matmul, data, x1, n, k)
    assert np.array_equal(after.view(np.uint32), before.view(np.uint32))
    lib.clq_clear_cache()


def test_forget_then_new_bytes_at_the_same_address(cuda, clq, synth, oracle):
    lib = clq._lib.lib
    lib.clq_clear_cache()
    n, k = 128, 1024
    data = synth.packed_blocks("q4_k", n, k, seed=15)
    x = synth.activations(2, k, seed=33)
    old = call(lib, lib.clq_q4_k_matmul, data, x, n, k)
    assert np.array_equal(call(lib, lib.clq_q4_k_matmul, data, x, n, k).view(np.uint32), old.view(np.uint32))
    data[:] = synth.packed_blocks("q4_k", n, k, seed=16)  # same buffer, new weights
    stale = call(lib, lib.clq_q4_k_matmul, data, x, n, k)  # copy-once: still the old upload
    assert np.array_equal(stale.view(np.uint32), old.view(np.uint32))
    assert lib.clq_forget(data.ctypes.data, data.nbytes) == 0
    new = call(lib, lib.clq_q4_k_matmul, data, x, n, k)
    ref, mag = oracle.matmul_f64("q4_k", x, data, n)
    assert element_bound_ok(new, ref, mag)
    assert not np.array_equal(new, old)
    lib.clq_clear_cache()
