"""clq_linear_device_noalloc against clq_linear_device and the fp64 oracle (needs a B200).

The allocation-free entry point runs the tensor-core prefill GEMM with its
staging in the library's fixed device buffer.  Called through the C-ABI on two
different requests in a row, each result must agree with the allocating entry
point within the linear-output tolerance (the two may split K differently, so
the sums can round differently) and meet the GEMM's bounds against the fp64
oracle on a slice of weight rows; a repeated request must repeat its result
bit for bit whatever the buffer held before; a request too big for the buffer
must be refused before any device work.  This file sorts last so the buffer is
also exercised after the rest of the suite has run in the process.
"""
import ctypes

import numpy as np
import pytest

from helpers import NORM_REL, max_row_relative_error

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 << 20  # CLQ_NOALLOC_SCRATCH_BYTES


def lib(clq):
    from importlib import import_module
    return import_module(clq.__name__ + "._lib")


def noalloc(clq, store, x):
    torch = __import__("torch")
    _lib = lib(clq)
    m = x.shape[0]
    out = torch.full((m, store.n), float("nan"), dtype=torch.float32, device=x.device)
    xtype = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[x.dtype]
    _lib.check(_lib.lib.clq_linear_device_noalloc(store.handle, 0, store.n, x.data_ptr(), xtype, m,
                                                  out.data_ptr(), out.stride(0),
                                                  torch.cuda.current_stream().cuda_stream))
    return out


def agree(got, want):
    got = got.cpu().numpy()
    want = want.cpu().numpy()
    assert np.all(np.isfinite(got))
    assert max_row_relative_error(got, want.astype(np.float64)) <= NORM_REL


CASES = [
    # Llama-3-8B q/o projection, 512-token prompt: the allocating path splits K
    # four ways here, which would not fit, so this call splits it two ways
    ("q4_k", 4096, 4096, 512, "bfloat16"),
    # down projection with a ragged 100-token prompt, fp16 activations
    ("q6_k", 1024, 14336, 100, "float16"),
]


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls(cuda, clq, synth, oracle):
    torch = cuda
    for dtype, n, k, m, xt in CASES:
        data = synth.packed_blocks(dtype, n, k, seed=n + m)
        x = torch.from_numpy(synth.activations(m, k, seed=m)).cuda().to(getattr(torch, xt))
        store = clq.Store(dtype, n, k, data)
        got = noalloc(clq, store, x)
        want = store.linear(x)
        torch.cuda.synchronize()
        agree(got, want)
        # the fp64 oracle on the first 128 weight rows: the norm gate and the
        # GEMM's per-element bound for its two fp16 roundings
        rows = 128
        rb = k // clq.DTYPES[dtype].block_size * clq.DTYPES[dtype].block_bytes
        ref, mag = oracle.matmul_f64(dtype, x.float().cpu().numpy(), data[:rows * rb], rows)
        g = got.cpu().numpy()[:, :rows].astype(np.float64)
        assert max_row_relative_error(g, ref) <= NORM_REL
        assert np.all(np.abs(g - ref) <= 1e-3 * mag + 1e-6)
        store.close()


def test_noalloc_repeats_bit_for_bit(cuda, clq, synth):
    torch = cuda
    big = clq.Store("q4_0", 512, 2048, synth.packed_blocks("q4_0", 512, 2048, seed=1))
    small = clq.Store("q8_0", 256, 1024, synth.packed_blocks("q8_0", 256, 1024, seed=2))
    xb = torch.from_numpy(synth.activations(700, 2048, seed=3)).cuda().to(torch.bfloat16)
    xs = torch.from_numpy(synth.activations(64, 1024, seed=4)).cuda().to(torch.bfloat16)
    first = noalloc(clq, small, xs)
    noalloc(clq, big, xb)  # leaves other contents in the shared buffer
    second = noalloc(clq, small, xs)
    torch.cuda.synchronize()
    assert torch.equal(first, second)
    agree(second, small.linear(xs))
    big.close()
    small.close()


def test_noalloc_refuses_requests_beyond_its_buffer(cuda, clq, synth):
    torch = cuda
    _lib = lib(clq)
    n, k = 256, 14336
    store = clq.Store("q6_k", n, k, synth.packed_blocks("q6_k", n, k, seed=5))
    m = SCRATCH_BYTES // (2 * k) + 256  # the fp16 activation image alone overflows
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    rc = _lib.lib.clq_linear_device_noalloc(store.handle, 0, n, x.data_ptr(), 1, m, out.data_ptr(), n,
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 2  # CLQ_ERR_SHAPE
    assert "fixed buffer" in _lib.last_error()
    store.close()
