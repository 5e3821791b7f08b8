"""GGUF files as device stores (clq_gguf_*).

GGUFFile maps a GGUF v3 file and parses it in libclq with the reference
reader's checks (gguf/reader.lisp); malformed files raise ClqError with status
CLQ_ERR_FORMAT.  Tensor shapes are listed outermost first, as the reference's
tensor-info shape (gguf/reader.lisp:143: the file's dimensions reversed).
store(name) uploads a Q4_0 / Q8_0 / Q4_K / Q6_K tensor to the current device
(chunks read into page-locked staging, asynchronous copies; scales checked
and re-tiled on the device) and returns a Store; tensor_bytes(name) is the
tensor's bytes in the mapping, valid until close().
"""
import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from .store import Store


@dataclass(frozen=True)
class TensorInfo:
    name: str
    ggml_type: int
    shape: tuple   # outermost first
    offset: int    # in the data section
    nbytes: int


_STORE_DTYPE = {2: "q4_0", 8: "q8_0", 12: "q4_k", 14: "q6_k"}  # ggml type id -> packed dtype
_KIND = {0: "u8", 1: "i8", 2: "u16", 3: "i16", 4: "u32", 5: "i32", 6: "f32", 7: "bool", 8: "str",
         9: "array", 10: "u64", 11: "i64", 12: "f64"}


class GGUFFile:
    def __init__(self, path):
        handle = ctypes.c_void_p()
        _lib.check(_lib.lib.clq_gguf_open(str(path).encode(), ctypes.byref(handle)))
        self._handle = handle
        lib = _lib.lib
        count = ctypes.c_int64()
        _lib.check(lib.clq_gguf_tensor_count(handle, ctypes.byref(count)))
        self.tensors = {}
        for i in range(count.value):
            name, typ, rank = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
            dims = (ctypes.c_int64 * 4)()
            off, nb = ctypes.c_uint64(), ctypes.c_uint64()
            _lib.check(lib.clq_gguf_tensor_info(handle, i, ctypes.byref(name), ctypes.byref(typ), ctypes.byref(rank),
                                                dims, ctypes.byref(off), ctypes.byref(nb), None))
            shape = tuple(reversed([dims[d] for d in range(rank.value)]))
            key = name.value.decode()
            self.tensors[key] = TensorInfo(key, typ.value, shape, off.value, nb.value)
        _lib.check(lib.clq_gguf_metadata_count(handle, ctypes.byref(count)))
        self.keys = []
        for i in range(count.value):
            key = ctypes.c_char_p()
            _lib.check(lib.clq_gguf_metadata_key(handle, i, ctypes.byref(key), None))
            self.keys.append(key.value.decode())

    @property
    def handle(self):
        if self._handle is None:
            raise ValueError("GGUF file is closed")
        return self._handle

    def metadata(self, key):
        """A scalar or string value; for an array, ("array", element kind, length)."""
        t, u, i, f = ctypes.c_int(), ctypes.c_uint64(), ctypes.c_int64(), ctypes.c_double()
        s, slen, et, n = ctypes.c_char_p(), ctypes.c_uint64(), ctypes.c_int(), ctypes.c_uint64()
        _lib.check(_lib.lib.clq_gguf_metadata_value(self.handle, key.encode(), ctypes.byref(t), ctypes.byref(u),
                                                    ctypes.byref(i), ctypes.byref(f), ctypes.byref(s),
                                                    ctypes.byref(slen), ctypes.byref(et), ctypes.byref(n)))
        kind = _KIND[t.value]
        if kind in ("u8", "u16", "u32", "u64"):
            return u.value
        if kind in ("i8", "i16", "i32", "i64"):
            return i.value
        if kind in ("f32", "f64"):
            return f.value
        if kind == "bool":
            return bool(u.value)
        if kind == "str":
            return ctypes.string_at(s, slen.value).decode()
        return ("array", _KIND[et.value], n.value)

    def _index(self, name):
        idx = ctypes.c_int64()
        _lib.check(_lib.lib.clq_gguf_find_tensor(self.handle, name.encode(), ctypes.byref(idx)))
        return idx.value

    def tensor_bytes(self, name):
        """The tensor's bytes in the mapping (read-only uint8 array, valid until close())."""
        ptr = ctypes.c_void_p()
        nb = ctypes.c_uint64()
        _lib.check(_lib.lib.clq_gguf_tensor_info(self.handle, self._index(name), None, None, None, None, None,
                                                 ctypes.byref(nb), ctypes.byref(ptr)))
        if nb.value == 0:
            return np.zeros(0, np.uint8)
        arr = np.ctypeslib.as_array(ctypes.cast(ptr.value, ctypes.POINTER(ctypes.c_uint8)), shape=(nb.value,))
        arr.flags.writeable = False
        return arr

    def store(self, name):
        """The packed tensor NAME as a Store on the current device."""
        info = self.tensors[name]
        handle = ctypes.c_void_p()
        _lib.check(_lib.lib.clq_gguf_store(self.handle, self._index(name), ctypes.byref(handle)))
        rows = int(np.prod(info.shape[:-1])) if len(info.shape) > 1 else 1
        return Store.from_handle(_STORE_DTYPE[info.ggml_type], rows, info.shape[-1], handle)

    def close(self):
        if self._handle is not None:
            _lib.lib.clq_gguf_close(self._handle)
            self._handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
