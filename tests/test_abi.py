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
