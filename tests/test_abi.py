"""The C ABI library loads and exports what include/clq.h declares (CPU only).

Also the host-side argument checks that run before any device work.  On a
machine without a GPU, calls that need one report CLQ_ERR_NO_DEVICE rather
than falling back to the CPU.
"""
import ctypes
import pathlib
import re

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "clq.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(clq_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(clq):
    names = declared_functions()
    assert len(names) >= 20
    lib = clq._lib.lib
    for name in names:
        assert hasattr(lib, name), name
        assert name in clq._lib.SIGNATURES, f"{name} has no ctypes signature"


def test_python_binding_declares_only_header_symbols(clq):
    assert set(clq._lib.SIGNATURES) == set(declared_functions())


def test_abi_version_and_geometry(clq):
    lib = clq._lib.lib
    assert lib.clq_abi_version() == 1
    e, b = ctypes.c_int64(), ctypes.c_int64()
    for dtype, (ee, bb) in {2: (32, 18), 8: (32, 34), 12: (256, 144), 14: (256, 210)}.items():
        assert lib.clq_block_geometry(dtype, ctypes.byref(e), ctypes.byref(b)) == 0
        assert (e.value, b.value) == (ee, bb)
    assert lib.clq_block_geometry(3, ctypes.byref(e), ctypes.byref(b)) == 1
    assert "unknown packed dtype 3" in clq._lib.last_error()


def test_shape_errors_precede_device_work(clq):
    lib = clq._lib.lib
    out = np.zeros(4, np.float32)
    x = np.zeros(64, np.float32)
    w = np.zeros(2 * 144, np.uint8)
    # K not a multiple of the Q4_K block (gguf/reader.lisp:137-139)
    rc = lib.clq_q4_k_matmul(out.ctypes.data, x.ctypes.data, w.ctypes.data, 1, 2, 100)
    assert rc == 2 and "not a multiple of 256" in clq._lib.last_error()
    rc = lib.clq_matmul(99, out.ctypes.data, x.ctypes.data, w.ctypes.data, 1, 2, 256, 0)
    assert rc == 1
    # M = 0 is a no-op (tests/local/packed.lisp:53)
    assert lib.clq_q4_k_matmul(out.ctypes.data, x.ctypes.data, w.ctypes.data, 0, 2, 256) == 0
    # bytes that are not whole blocks (quant/q8-0.lisp:18-19)
    assert lib.clq_dequantize(8, w.ctypes.data, 35, out.ctypes.data) == 3


def test_calls_needing_a_device_fail_loudly_without_one(clq):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = clq._lib.lib
    out = np.zeros(2, np.float32)
    x = np.zeros(256, np.float32)
    w = np.zeros(2 * 144, np.uint8)
    rc = lib.clq_q4_k_matmul(out.ctypes.data, x.ctypes.data, w.ctypes.data, 1, 2, 256)
    assert rc == 8, clq._lib.last_error()
    with pytest.raises(clq.ClqError) as err:
        clq.linear(x.reshape(1, 256), clq.make_tensor_view(clq.make_q4_k_storage(w), (2, 256)))
    assert err.value.status == "CLQ_ERR_NO_DEVICE"
    status = ctypes.c_int(-1)
    assert lib.clq_device_status(ctypes.byref(status)) == 8
    assert status.value == 0


def test_cache_starts_empty_and_forget_is_safe(clq):
    lib = clq._lib.lib
    n, b = ctypes.c_int64(), ctypes.c_int64()
    assert lib.clq_clear_cache() == 0
    assert lib.clq_cache_stats(ctypes.byref(n), ctypes.byref(b)) == 0
    assert (n.value, b.value) == (0, 0)
    assert lib.clq_forget(None, 0) == 0


def test_kv_cache_rope_and_attention_argument_checks(clq):
    """The cache, RoPE and attention entry points reject bad arguments before
    any device work (so these run without a GPU)."""
    lib = clq._lib.lib
    out = ctypes.c_void_p()
    assert lib.clq_kv_cache_create(0, 1, 1, 8, 0, ctypes.byref(out)) == 2      # no positions
    assert lib.clq_kv_cache_create(4, 1, 1, 8, 7, ctypes.byref(out)) == 1      # unknown cache type
    assert "unknown cache type 7" in clq._lib.last_error()
    assert lib.clq_kv_cache_create(4, 1, 1, 8, 0, None) == 1
    assert lib.clq_kv_cache_destroy(None) == 0
    assert lib.clq_kv_cache_info(None, None, None, None, None, None) == 1
    assert lib.clq_kv_cache_update(None, 0, None, None, 1, 8, 8, 0, None) == 1
    status = ctypes.c_int()
    assert lib.clq_kv_cache_status(None, ctypes.byref(status)) == 1
    assert lib.clq_kv_cache_read(None, 0, 1, None, None, None) == 1
    assert lib.clq_attend_device(None, 1, 4, 32, None, 0, 1, 0, None, 32, None) == 1
    fake = 256  # a non-null address that the checks below never reach
    rope = lib.clq_rope_device
    assert rope(fake, 1, 2, 8, 16, 8, 7, 0, 10000.0, None, 0, None) == 2      # odd rotated width
    assert rope(fake, 1, 2, 8, 16, 8, 10, 0, 10000.0, None, 0, None) == 2     # wider than the head
    assert rope(fake, 1, 2, 8, 16, 8, 8, 0, 10000.0, None, 5, None) == 1      # unknown pairing
    assert rope(fake, 1, 2, 8, 16, 8, 8, 0, 0.0, None, 0, None) == 1          # theta must be positive
    assert rope(fake, 1, 2, 8, 8, 4, 8, 0, 10000.0, None, 0, None) == 2       # heads overlap
    assert rope(fake, 3, 2, 8, 8, 16, 8, 0, 10000.0, None, 0, None) == 2      # positions overlap heads
    # positions inside each head (a transposed layout) pass the checks: without a
    # GPU the call then fails as such (with one it would launch on the fake
    # address, so it is made only when no device is present)
    import torch
    if not torch.cuda.is_available():
        rc = rope(fake, 3, 2, 8, 8, 24, 8, 0, 10000.0, None, 0, None)
        assert rc == 8, clq._lib.last_error()
    assert rope(None, 0, 2, 8, 16, 8, 8, 0, 10000.0, None, 0, None) == 0      # no rows: nothing to do
    assert rope(None, 1, 2, 8, 16, 8, 8, 0, 10000.0, None, 0, None) == 1      # null rows


def test_kv_cache_needs_a_device(clq):
    import importlib

    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    att = importlib.import_module("cl-inference_b200.attention")
    with pytest.raises(clq.ClqError) as err:
        att.KVCache(16, 1, 2, 8)
    assert err.value.status == "CLQ_ERR_NO_DEVICE"
    with pytest.raises(clq.ClqError):
        att.KVCache(16, 1, 2, 8, "q4")
