"""B200 (sm_100a) quantized-linear path for cl-inference's packed GGUF weights.

Host-side mirror of cl-inference's packed-weight API (quant/packed.lisp,
quant/q8-0.lisp) over libclq.so, the CUDA library behind include/clq.h.
Importing fails if libclq.so has not been built: there is no CPU path.
"""
from . import _lib
from ._lib import ClqError
from .quant import (DTYPES, PackedDtype, PackedError, PackedStorage, PackedTensor,
                    UnsupportedOperation, astype, copy_tensor, dequantize, find_dtype, linear,
                    make_packed_storage, make_q4_0_storage, make_q4_k_storage, make_q6_k_storage,
                    make_q8_0_storage, make_tensor_view, matmul, slice_rows, take, take_dequantized,
                    transpose)
from .store import Store, linear_fused, linear_group, linear_group_fused

__all__ = [
    "ClqError", "DTYPES", "PackedDtype", "PackedError", "PackedStorage", "PackedTensor", "Store",
    "UnsupportedOperation", "astype", "copy_tensor", "dequantize", "find_dtype", "linear",
    "make_packed_storage", "make_q4_0_storage", "make_q4_k_storage", "make_q6_k_storage",
    "make_q8_0_storage", "make_tensor_view", "matmul", "slice_rows", "take", "take_dequantized",
    "transpose", "linear_group",
]
