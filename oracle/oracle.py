"""ctypes wrapper of the CPU oracle (libclq_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker.  Never imported by the product.
The C source (clq_oracle.c) cites the cl-inference lines each function follows.
"""
import ctypes
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIBRARY_PATH = HERE / "libclq_oracle.so"

Q4_0, Q8_0, Q4_K, Q6_K = 2, 8, 12, 14
GGML = {"q4_0": Q4_0, "q8_0": Q8_0, "q4_k": Q4_K, "q6_k": Q6_K}
OK, ERR_ARGUMENT, ERR_NONFINITE = 0, 1, 4


def build():
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _load():
    if not LIBRARY_PATH.exists():
        build()
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    p, i64, i = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.clqo_block_geometry.argtypes = [i, ctypes.POINTER(i64), ctypes.POINTER(i64)]
    lib.clqo_block_scale.argtypes = [ctypes.c_uint8, ctypes.c_uint8, ctypes.POINTER(ctypes.c_float)]
    lib.clqo_element.argtypes = [i, p, i, ctypes.POINTER(ctypes.c_float)]
    lib.clqo_dequantize.argtypes = [i, p, i64, p, ctypes.POINTER(i64)]
    lib.clqo_gather.argtypes = [i, p, i64, i64, p, i64, p]
    lib.clqo_matmul_f64.argtypes = [i, p, p, i64, i64, i64, p, p, i]
    lib.clqo_matmul_f32.argtypes = [i, p, p, i64, i64, i64, p, i]
    lib.clqo_max_threads.argtypes = []
    return lib


lib = _load()


class OracleError(ValueError):
    def __init__(self, code, what):
        self.code = code
        super().__init__(f"oracle status {code}: {what}")


def _dtype(dtype):
    return GGML[dtype] if isinstance(dtype, str) else int(dtype)


def geometry(dtype):
    e, b = ctypes.c_int64(), ctypes.c_int64()
    if not lib.clqo_block_geometry(_dtype(dtype), ctypes.byref(e), ctypes.byref(b)):
        raise OracleError(ERR_ARGUMENT, f"unknown dtype {dtype}")
    return e.value, b.value


def block_scale(low, high):
    out = ctypes.c_float()
    rc = lib.clqo_block_scale(low, high, ctypes.byref(out))
    if rc:
        raise OracleError(rc, "Quantized scale is not finite")
    return np.float32(out.value)


def dequantize(dtype, data):
    """f32 values of every block in DATA (bytes or uint8 array)."""
    e, b = geometry(dtype)
    data = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8) if isinstance(data, (bytes, bytearray))
                                else data, dtype=np.uint8)
    nblocks = data.size // b
    out = np.empty(nblocks * e, dtype=np.float32)
    bad = ctypes.c_int64(-1)
    rc = lib.clqo_dequantize(_dtype(dtype), data.ctypes.data, nblocks, out.ctypes.data, ctypes.byref(bad))
    if rc:
        raise OracleError(rc, f"block {bad.value}")
    return out


def gather(dtype, data, n, k, ids):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.empty((ids.size, k), dtype=np.float32)
    rc = lib.clqo_gather(_dtype(dtype), data.ctypes.data, n, k, ids.ctypes.data, ids.size, out.ctypes.data)
    if rc:
        raise OracleError(rc, "gather")
    return out


def matmul_f64(dtype, x, data, n, threads=0):
    """(sum, magnitude): fp64 x . dequant(W)^T and sum |x*w| per output."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    out = np.empty((m, n), dtype=np.float64)
    mag = np.empty((m, n), dtype=np.float64)
    rc = lib.clqo_matmul_f64(_dtype(dtype), x.ctypes.data, data.ctypes.data, m, n, k, out.ctypes.data,
                             mag.ctypes.data, threads)
    if rc:
        raise OracleError(rc, "matmul_f64")
    return out, mag


def matmul_f32(dtype, x, data, n, threads=0):
    """fp32 port of the CPU kernel contract (the timed CPU baseline)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    out = np.empty((m, n), dtype=np.float32)
    rc = lib.clqo_matmul_f32(_dtype(dtype), x.ctypes.data, data.ctypes.data, m, n, k, out.ctypes.data,
                             threads)
    if rc:
        raise OracleError(rc, "matmul_f32")
    return out


def max_threads():
    return lib.clqo_max_threads()
