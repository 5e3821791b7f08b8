"""Block geometry of the packed GGUF dtypes, with no dependency on libclq.so.

The ggml type ids and block shapes are fixed by the file format
(gguf/reader.lisp:37-52) and registered by quant/q8-0.lisp:5-6 and
quant/packed.lisp:156-158 of cl-inference.  Kept apart from quant.py so that
shape arithmetic (tensor-parallel plans, synthetic weights) imports without
loading the CUDA library.
"""
from dataclasses import dataclass


class UnsupportedOperation(TypeError):
    """ct:unsupported-operation: no executor resolves (quant/packed.lisp:126-139)."""


@dataclass(frozen=True)
class PackedDtype:
    name: str
    ggml_type: int
    block_size: int
    block_bytes: int


DTYPES = {
    "q8_0": PackedDtype("q8_0", 8, 32, 34),
    "q4_0": PackedDtype("q4_0", 2, 32, 18),
    "q4_k": PackedDtype("q4_k", 12, 256, 144),
    "q6_k": PackedDtype("q6_k", 14, 256, 210),
}
BY_GGML_TYPE = {d.ggml_type: d for d in DTYPES.values()}


def find_dtype(dtype):
    if isinstance(dtype, PackedDtype):
        return dtype
    try:
        return DTYPES[str(dtype).lower().lstrip(":")]
    except KeyError:
        raise UnsupportedOperation(f"{dtype!r} is not a packed dtype") from None
