"""ctypes binding of libclq.so (include/clq.h).

Loading fails loudly when the shared library is missing: there is no CPU path
behind this package.
"""
import ctypes
import os
import pathlib

_HERE = pathlib.Path(__file__).resolve().parent
LIBRARY_PATH = _HERE / "libclq.so"

CLQ_Q4_0, CLQ_Q8_0, CLQ_Q4_K, CLQ_Q6_K = 2, 8, 12, 14
CLQ_X_F32, CLQ_X_BF16, CLQ_X_F16 = 0, 1, 2
CLQ_MATH_DEFAULT, CLQ_MATH_FAST, CLQ_NO_CACHE, CLQ_MATH_EXACT = 0, 1, 2, 4

STATUS_NAMES = {
    0: "CLQ_OK", 1: "CLQ_ERR_ARGUMENT", 2: "CLQ_ERR_SHAPE", 3: "CLQ_ERR_BLOCKS",
    4: "CLQ_ERR_NONFINITE_SCALE", 5: "CLQ_ERR_CUDA", 6: "CLQ_ERR_NCCL", 7: "CLQ_ERR_TIMEOUT",
    8: "CLQ_ERR_NO_DEVICE", 9: "CLQ_ERR_UNSUPPORTED", 10: "CLQ_ERR_OUT_OF_MEMORY",
    11: "CLQ_ERR_FORMAT", 12: "CLQ_ERR_IO", 13: "CLQ_ERR_NONFINITE_VALUE", 14: "CLQ_ERR_CONTEXT",
}

_i64 = ctypes.c_int64
_u32 = ctypes.c_uint
_ptr = ctypes.c_void_p
_int = ctypes.c_int
_size = ctypes.c_size_t

# name -> (restype, argtypes); every symbol include/clq.h declares.
SIGNATURES = {
    "clq_abi_version": (_int, []),
    "clq_last_error": (_int, [ctypes.c_char_p, _size]),
    "clq_device_status": (_int, [_ptr]),
    "clq_block_geometry": (_int, [_int, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "clq_q8_0_matmul": (_int, [_ptr, _ptr, _ptr, _i64, _i64, _i64]),
    "clq_q4_0_matmul": (_int, [_ptr, _ptr, _ptr, _i64, _i64, _i64]),
    "clq_q4_k_matmul": (_int, [_ptr, _ptr, _ptr, _i64, _i64, _i64]),
    "clq_q6_k_matmul": (_int, [_ptr, _ptr, _ptr, _i64, _i64, _i64]),
    "clq_matmul": (_int, [_int, _ptr, _ptr, _ptr, _i64, _i64, _i64, _u32]),
    "clq_forget": (_int, [_ptr, _size]),
    "clq_clear_cache": (_int, []),
    "clq_cache_stats": (_int, [ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "clq_store_create": (_int, [_int, _i64, _i64, _ptr, _size, _u32, ctypes.POINTER(_ptr)]),
    "clq_store_create_device": (_int, [_int, _i64, _i64, _ptr, _size, _u32, _ptr, ctypes.POINTER(_ptr)]),
    "clq_store_free": (_int, [_ptr]),
    "clq_store_info": (_int, [_ptr, ctypes.POINTER(_int), ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                              ctypes.POINTER(_size), ctypes.POINTER(_ptr), ctypes.POINTER(_int)]),
    "clq_linear_device": (_int, [_ptr, _i64, _i64, _ptr, _int, _i64, _ptr, _i64, _u32, _ptr]),
    "clq_linear_group_device": (_int, [_ptr, _ptr, _ptr, _int, _ptr, _int, _i64, _ptr, _ptr, _u32, _ptr]),
    "clq_linear_device_noalloc": (_int, [_ptr, _i64, _i64, _ptr, _int, _i64, _ptr, _i64, _ptr]),
    "clq_tp_buffers": (_int, [_int, _i64, ctypes.POINTER(_ptr), ctypes.POINTER(_ptr)]),
    "clq_tp_buffers_free": (_int, [_ptr, _ptr]),
    "clq_ipc_handle": (_int, [_ptr, _ptr]),
    "clq_ipc_open": (_int, [_ptr, ctypes.POINTER(_ptr)]),
    "clq_ipc_close": (_int, [_ptr]),
    "clq_linear_fused_device": (_int, [_ptr, _i64, _i64, _ptr, _int, _i64, _ptr, _ptr, _i64, ctypes.c_uint, _ptr]),
    "clq_linear_group_fused_device": (_int, [ctypes.POINTER(_ptr), ctypes.POINTER(_i64), ctypes.POINTER(_i64), _int,
                                             _ptr, _int, _i64, _ptr, ctypes.POINTER(_ptr), ctypes.POINTER(_i64),
                                             ctypes.c_uint, _ptr]),
    "clq_gguf_open": (_int, [ctypes.c_char_p, _ptr]),
    "clq_gguf_close": (_int, [_ptr]),
    "clq_gguf_tensor_count": (_int, [_ptr, ctypes.POINTER(_i64)]),
    "clq_gguf_tensor_info": (_int, [_ptr, _i64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_int),
                                    ctypes.POINTER(_int), ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_uint64),
                                    ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_ptr)]),
    "clq_gguf_find_tensor": (_int, [_ptr, ctypes.c_char_p, ctypes.POINTER(_i64)]),
    "clq_gguf_metadata_count": (_int, [_ptr, ctypes.POINTER(_i64)]),
    "clq_gguf_metadata_key": (_int, [_ptr, _i64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_int)]),
    "clq_gguf_metadata_value": (_int, [_ptr, ctypes.c_char_p, ctypes.POINTER(_int), ctypes.POINTER(ctypes.c_uint64),
                                       ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_double),
                                       ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_uint64),
                                       ctypes.POINTER(_int), ctypes.POINTER(ctypes.c_uint64)]),
    "clq_gguf_store": (_int, [_ptr, _i64, _ptr]),
    "clq_tp_create": (_int, [_int, _int, _i64, _ptr, _ptr, ctypes.POINTER(_ptr)]),
    "clq_tp_free": (_int, [_ptr]),
    "clq_linear_allreduce_device": (_int, [_ptr, _i64, _i64, _ptr, _int, _i64, _ptr, _i64, _ptr, _ptr]),
    "clq_dequantize_device": (_int, [_ptr, _i64, _i64, _ptr, _int, _ptr]),
    "clq_gather_device": (_int, [_ptr, _ptr, _i64, _ptr, _ptr]),
    "clq_dequantize": (_int, [_int, _ptr, _size, _ptr]),
    "clq_take": (_int, [_int, _ptr, _i64, _i64, _ptr, _i64, _ptr]),
    "clq_kv_cache_create": (_int, [_i64, _int, _int, _int, _int, ctypes.POINTER(_ptr)]),
    "clq_kv_cache_destroy": (_int, [_ptr]),
    "clq_kv_cache_info": (_int, [_ptr, ctypes.POINTER(_i64), ctypes.POINTER(_int), ctypes.POINTER(_int),
                                 ctypes.POINTER(_int), ctypes.POINTER(_int)]),
    "clq_kv_cache_update": (_int, [_ptr, _int, _ptr, _ptr, _i64, _i64, _i64, _i64, _ptr]),
    "clq_kv_cache_status": (_int, [_ptr, ctypes.POINTER(_int)]),
    "clq_kv_cache_read": (_int, [_ptr, _int, _i64, _ptr, _ptr, _ptr]),
    "clq_rope_device": (_int, [_ptr, _i64, _int, _int, _i64, _i64, _int, _i64, ctypes.c_double, _ptr, _int, _ptr]),
    "clq_attend_device": (_int, [_ptr, _i64, _int, _i64, _ptr, _int, _i64, _i64, _ptr, _i64, _ptr]),
}


class ClqError(RuntimeError):
    """A non-zero status from libclq, with the library's message."""

    def __init__(self, code, message):
        self.code = code
        self.status = STATUS_NAMES.get(code, str(code))
        super().__init__(f"{self.status}: {message}")


def load(path=None):
    path = pathlib.Path(path or os.environ.get("CLQ_LIBRARY", LIBRARY_PATH))
    if not path.exists():
        raise ImportError(f"libclq.so not built at {path}; run __graft_entry__.build()")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = load()


def last_error():
    buf = ctypes.create_string_buffer(1024)
    lib.clq_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc):
    if rc != 0:
        raise ClqError(rc, last_error())
    return rc
