"""Packed GGUF dtypes (Q8_0, Q4_0, Q4_K, Q6_K) with cl-inference's packed-weight API.

Mirrors quant/packed.lisp and quant/q8-0.lisp of cl-inference: storage over
whole blocks, the view rules, `matmul` of f32 activations by a transposed
packed weight, dequantize, take and copy.  The arithmetic runs in libclq.so on
the GPU; this module only validates, views and moves host buffers.
Paths in docstrings are relative to the cl-inference project.
"""
import weakref

import numpy as np

from . import _lib
# the dtypes of quant/q8-0.lisp:5-6 and the registrations of quant/packed.lisp:156-158
from .geometry import BY_GGML_TYPE, DTYPES, PackedDtype, UnsupportedOperation, find_dtype  # noqa: F401


class PackedError(ValueError):
    """The reference's Lisp `error` for bad storage, views or copies."""


assert all(getattr(_lib, "CLQ_" + d.name.upper()) == d.ggml_type for d in DTYPES.values())


class PackedStorage:
    """Bytes of whole blocks (make-packed-storage, quant/packed.lisp:11-17).

    DATA is a 1-D uint8 numpy array: an owned vector or a zero-copy view over a
    mapping.  When this object is collected, the device copy libclq cached for
    its address range is dropped (the close-weights hook of the C ABI).
    """

    def __init__(self, dtype, data):
        dtype = find_dtype(dtype)
        if not (isinstance(data, np.ndarray) and data.dtype == np.uint8 and data.ndim == 1
                and data.flags.c_contiguous):
            raise PackedError("Packed storage requires simple unsigned byte vectors or views")
        if data.size % dtype.block_bytes:
            raise PackedError(f"{dtype.name} data of {data.size} bytes is not a whole number of blocks")
        self.dtype = dtype
        self.bytes = data
        self._finalizer = weakref.finalize(self, _forget, data.ctypes.data, data.size)

    @property
    def storage_length(self):
        """ct:storage-length: elements held (quant/packed.lisp:19-21)."""
        return self.dtype.block_size * (self.bytes.size // self.dtype.block_bytes)


def _forget(address, nbytes):
    try:
        _lib.lib.clq_forget(address, nbytes)
    except Exception:  # interpreter shutdown
        pass


def make_packed_storage(dtype, data):
    if isinstance(data, (bytes, bytearray)):
        data = np.frombuffer(bytes(data), dtype=np.uint8).copy()
    return PackedStorage(dtype, data)


def make_q8_0_storage(data): return make_packed_storage("q8_0", data)
def make_q4_0_storage(data): return make_packed_storage("q4_0", data)
def make_q4_k_storage(data): return make_packed_storage("q4_k", data)
def make_q6_k_storage(data): return make_packed_storage("q6_k", data)


def _row_major_strides(shape):
    strides, acc = [], 1
    for size in reversed(shape):
        strides.append(acc)
        acc *= size
    return tuple(reversed(strides))


class PackedTensor:
    """A validated view of packed storage: whole rows of blocks, or their transpose."""

    def __init__(self, storage, shape, strides, offset):
        self.storage, self.shape, self.strides, self.offset = storage, tuple(shape), tuple(strides), offset

    @property
    def dtype(self):
        return self.storage.dtype

    @property
    def size(self):
        return int(np.prod(self.shape)) if self.shape else 1

    def row_major_p(self):
        return self.strides == _row_major_strides(self.shape)

    def transposed_matrix_p(self):
        """quant/q8-0.lisp:56-58: the transpose of a row-major matrix."""
        return len(self.shape) == 2 and self.strides[0] == 1 and self.shape[0] == self.strides[1]

    def byte_offset(self):
        """packed-byte-offset, quant/packed.lisp:42-44."""
        return (self.offset // self.dtype.block_size) * self.dtype.block_bytes


def make_tensor_view(storage, shape, offset=0, strides=None):
    """ct:make-tensor-view with validate-storage-view (quant/packed.lisp:30-40)."""
    shape = tuple(int(s) for s in shape)
    strides = _row_major_strides(shape) if strides is None else tuple(strides)
    t = PackedTensor(storage, shape, strides, int(offset))
    e = storage.dtype.block_size
    ok = (offset % e == 0 and len(shape) > 0
          and ((t.row_major_p() and shape[-1] % e == 0)
               or (t.transposed_matrix_p() and shape[0] % e == 0)))
    if not ok:
        raise PackedError(f"{storage.dtype.name} views require whole packed rows or their transpose")
    reach = offset + sum((s - 1) * st for s, st in zip(shape, strides)) + 1 if t.size else offset
    if reach > storage.storage_length:
        raise PackedError(f"view reaches element {reach} of {storage.storage_length}")
    return t


def transpose(t):
    if len(t.shape) != 2:
        raise UnsupportedOperation("transpose needs a matrix")
    return PackedTensor(t.storage, t.shape[::-1], t.strides[::-1], t.offset)


def slice_rows(t, start, end):
    """Rows [start, end) of a row-major view (ct:slice on the first axis)."""
    if not t.row_major_p():
        raise PackedError("row slices need a row-major view")
    return make_tensor_view(t.storage, (end - start,) + t.shape[1:], t.offset + start * t.strides[0])


def packed_weight_bytes(t):
    """Bytes from the view's whole-row offset on (quant/packed.lisp:60-66)."""
    return t.storage.bytes[t.byte_offset():]


def _as_f32_matrix(x):
    x = np.asarray(x)
    if x.dtype != np.float32 or x.ndim != 2:
        return None
    return np.ascontiguousarray(x)  # the executor copies a non-contiguous x (packed.lisp:71)


def matmul(x, weight, flags=0):
    """x[M,K] . weight for a transposed packed (K N) view: f32 [M, N].

    resolve-operation :matmul (quant/packed.lisp:128-135, quant/q8-0.lisp:127-132)
    then the executor (packed.lisp:68-75 / q8-0.lisp:77-85), which calls the
    6-argument kernel; here that kernel is libclq's clq_matmul.
    """
    if not isinstance(weight, PackedTensor):
        raise UnsupportedOperation("matmul needs a packed weight on the right")
    xs = _as_f32_matrix(x)
    if (xs is None or not weight.transposed_matrix_p() or xs.shape[1] != weight.shape[0]
            or (weight.dtype.name == "q8_0" and weight.offset != 0)):
        raise UnsupportedOperation(
            f"no {weight.dtype.name} matmul for x {getattr(x, 'shape', None)} and weight {weight.shape}")
    m, k = xs.shape
    n = weight.shape[1]
    out = np.empty((m, n), dtype=np.float32)
    if m == 0 or n == 0:
        return out
    wb = packed_weight_bytes(weight)
    _lib.check(_lib.lib.clq_matmul(weight.dtype.ggml_type, out.ctypes.data, xs.ctypes.data,
                                   wb.ctypes.data, m, n, k, flags))
    return out


def linear(x, weight, flags=0):
    """X . WEIGHT^T for a packed (out in) weight (local/blocks.lisp:106-113)."""
    return matmul(x, transpose(weight), flags)


def _dequantize_blocks(dtype, data):
    out = np.empty(data.size // dtype.block_bytes * dtype.block_size, dtype=np.float32)
    if out.size:
        _lib.check(_lib.lib.clq_dequantize(dtype.ggml_type, data.ctypes.data, data.size, out.ctypes.data))
    return out


def dequantize(t):
    """ct:dequantize / ct:astype :f32 of a packed view (quant/packed.lisp:110-124)."""
    e = t.dtype.block_size
    if t.row_major_p():
        rows = t.size // t.shape[-1] if t.size else 0
        first = t.byte_offset()
        nbytes = t.size // e * t.dtype.block_bytes
        flat = _dequantize_blocks(t.dtype, t.storage.bytes[first:first + nbytes])
        return flat.reshape(t.shape) if rows else np.empty(t.shape, np.float32)
    if t.transposed_matrix_p():
        return dequantize(transpose(t)).T.copy()
    raise PackedError("packed views are row-major or transposed matrices")


def astype(t, dtype):
    if str(dtype).lower().lstrip(":") != "f32":
        raise UnsupportedOperation(f"no packed conversion to {dtype}")
    return dequantize(t)


def take(t, ids):
    """ct:take of rows: the rows keep the packed dtype, duplicates allowed."""
    if len(t.shape) != 2 or not t.row_major_p():
        raise UnsupportedOperation("take needs a row-major packed matrix")
    ids = np.asarray(ids, dtype=np.int64).ravel()
    if ids.size and (ids.min() < 0 or ids.max() >= t.shape[0]):
        raise PackedError("take index out of range")
    row_bytes = t.shape[1] // t.dtype.block_size * t.dtype.block_bytes
    base = packed_weight_bytes(t)
    rows = [base[i * row_bytes:(i + 1) * row_bytes] for i in ids]
    data = np.concatenate(rows) if rows else np.empty(0, np.uint8)
    return make_tensor_view(PackedStorage(t.dtype, data.copy()), (ids.size, t.shape[1]))


def take_dequantized(t, ids):
    """Rows IDS of a row-major packed matrix as f32, gathered on the device."""
    if len(t.shape) != 2 or not t.row_major_p():
        raise UnsupportedOperation("take needs a row-major packed matrix")
    ids32 = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).ravel())
    out = np.empty((ids32.size, t.shape[1]), dtype=np.float32)
    if out.size:
        wb = packed_weight_bytes(t)
        _lib.check(_lib.lib.clq_take(t.dtype.ggml_type, wb.ctypes.data, t.shape[0], t.shape[1],
                                     ids32.ctypes.data, ids32.size, out.ctypes.data))
    return out


def copy_tensor(t):
    """ct:copy-tensor: packed bytes copied without upcast (quant/packed.lisp:49-58)."""
    if not t.row_major_p():
        raise PackedError("Packed copies require contiguous tensors of one dtype and shape")
    first = t.byte_offset()
    nbytes = t.size // t.dtype.block_size * t.dtype.block_bytes
    data = t.storage.bytes[first:first + nbytes].copy()
    return make_tensor_view(PackedStorage(t.dtype, data), t.shape)
