"""Device-resident packed-weight store and device-pointer products.

torch provides device memory and streams here (plumbing); the products,
dequantize and gather are libclq kernels.
"""
import ctypes

import numpy as np

from . import _lib
from .quant import find_dtype

_XTYPE = {"float32": _lib.CLQ_X_F32, "bfloat16": _lib.CLQ_X_BF16, "float16": _lib.CLQ_X_F16}


def _torch():
    import torch
    return torch


def current_stream_handle():
    torch = _torch()
    return torch.cuda.current_stream().cuda_stream


class Store:
    """N x K packed blocks uploaded once in native GGUF layout (clq_store_create).

    DATA is a host uint8 numpy array, or a uint8 CUDA tensor on the current device.
    """

    def __init__(self, dtype, n, k, data):
        self.dtype = find_dtype(dtype)
        self.n, self.k = int(n), int(k)
        handle = ctypes.c_void_p()
        torch = _torch()
        if isinstance(data, np.ndarray):
            data = np.ascontiguousarray(data, dtype=np.uint8)
            _lib.check(_lib.lib.clq_store_create(self.dtype.ggml_type, self.n, self.k, data.ctypes.data,
                                                 data.size, 0, ctypes.byref(handle)))
        elif isinstance(data, torch.Tensor) and data.is_cuda and data.dtype == torch.uint8:
            data = data.contiguous()
            _lib.check(_lib.lib.clq_store_create_device(self.dtype.ggml_type, self.n, self.k,
                                                        data.data_ptr(), data.numel(), 0,
                                                        current_stream_handle(), ctypes.byref(handle)))
        else:
            raise TypeError("store data must be a uint8 numpy array or a uint8 CUDA tensor")
        self._handle = handle

    @classmethod
    def from_handle(cls, dtype, n, k, handle):
        """Wrap a clq_store made elsewhere (clq_gguf_store); the Store owns it."""
        self = cls.__new__(cls)
        self.dtype = find_dtype(dtype)
        self.n, self.k = int(n), int(k)
        self._handle = handle
        return self

    @property
    def handle(self):
        if self._handle is None:
            raise ValueError("store is closed")
        return self._handle

    @property
    def row_bytes(self):
        return self.k // self.dtype.block_size * self.dtype.block_bytes

    def close(self):
        if self._handle is not None:
            _lib.lib.clq_store_free(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def linear(self, x, out=None, row_begin=0, rows=None, flags=0, stream=None):
        """out[m, :rows] = x[m, K] . W[row_begin:row_begin+rows]^T (clq_linear_device)."""
        torch = _torch()
        rows = self.n - row_begin if rows is None else rows
        if x.dim() != 2 or x.shape[1] != self.k or not x.is_cuda:
            raise ValueError(f"x must be a CUDA [m, {self.k}] matrix, got {tuple(x.shape)}")
        x = x.contiguous()
        m = x.shape[0]
        if out is None:
            out = torch.empty((m, rows), dtype=torch.float32, device=x.device)
        ldo = out.stride(0) if out.dim() == 2 and m > 0 else rows
        if out.dtype != torch.float32 or (out.dim() == 2 and out.stride(1) != 1):
            raise ValueError("out must be float32 with unit column stride")
        xtype = _XTYPE.get(str(x.dtype).replace("torch.", ""))
        if xtype is None:
            raise ValueError(f"unsupported activation dtype {x.dtype}")
        _lib.check(_lib.lib.clq_linear_device(self.handle, row_begin, rows, x.data_ptr(), xtype, m,
                                              out.data_ptr(), ldo, flags,
                                              stream if stream is not None else current_stream_handle()))
        return out

    def dequantize(self, row_begin=0, rows=None, transposed=False, out=None):
        torch = _torch()
        rows = self.n - row_begin if rows is None else rows
        if out is None:
            shape = (self.k, rows) if transposed else (rows, self.k)
            out = torch.empty(shape, dtype=torch.float32, device="cuda")
        _lib.check(_lib.lib.clq_dequantize_device(self.handle, row_begin, rows, out.data_ptr(),
                                                  1 if transposed else 0, current_stream_handle()))
        return out

    def gather(self, ids, out=None):
        torch = _torch()
        ids = ids.to(dtype=torch.int32).contiguous()
        if out is None:
            out = torch.empty((ids.numel(), self.k), dtype=torch.float32, device=ids.device)
        _lib.check(_lib.lib.clq_gather_device(self.handle, ids.data_ptr(), ids.numel(), out.data_ptr(),
                                              current_stream_handle()))
        return out


class _Fusion(ctypes.Structure):
    _fields_ = [("norm_weight", ctypes.c_void_p), ("norm_epsilon", ctypes.c_float), ("gate", ctypes.c_void_p),
                ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64)]


def _fusion(x, norm_weight, eps, gate, residual):
    """The clq_fusion of the optional fp32 [K] NORM_WEIGHT, GATE (x's type and
    shape) and fp32 RESIDUAL; the tensors are returned to keep them alive."""
    torch = _torch()
    keep = []
    f = _Fusion(None, float(eps), None, None, 0)
    if norm_weight is not None:
        norm_weight = norm_weight.to(device=x.device, dtype=torch.float32).contiguous()
        if norm_weight.numel() != x.shape[1]:
            raise ValueError(f"norm weight has {norm_weight.numel()} elements for rows of {x.shape[1]}")
        f.norm_weight = norm_weight.data_ptr()
        keep.append(norm_weight)
    if gate is not None:
        if gate.shape != x.shape or gate.dtype != x.dtype or not gate.is_cuda:
            raise ValueError("gate must match x's shape, type and device")
        gate = gate.contiguous()
        f.gate = gate.data_ptr()
        keep.append(gate)
    if residual is not None:
        if residual.dtype != torch.float32 or residual.dim() != 2 or residual.stride(1) != 1:
            raise ValueError("residual must be an fp32 [m, n] matrix with unit column stride")
        f.residual = residual.data_ptr()
        f.ldr = residual.stride(0)
        keep.append(residual)
    return f, keep


def linear_fused(store, x, out=None, norm_weight=None, eps=1e-5, gate=None, residual=None, row_begin=0, rows=None,
                 flags=0, stream=None):
    """out = h(x) . W^T (+ residual) with the RMSNorm / SwiGLU prologue and the
    residual epilogue of clq_linear_fused_device."""
    torch = _torch()
    rows = store.n - row_begin if rows is None else rows
    x = x.contiguous()
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, rows), dtype=torch.float32, device=x.device)
    f, keep = _fusion(x, norm_weight, eps, gate, residual)
    xtype = _XTYPE.get(str(x.dtype).replace("torch.", ""))
    _lib.check(_lib.lib.clq_linear_fused_device(store.handle, row_begin, rows, x.data_ptr(), xtype, m,
                                                ctypes.byref(f), out.data_ptr(), out.stride(0), flags,
                                                stream if stream is not None else current_stream_handle()))
    del keep
    return out


def linear_group_fused(stores, x, norm_weight=None, eps=1e-5, gate=None, outs=None, flags=0, stream=None):
    """linear_group over the fused input h(x) (clq_linear_group_fused_device)."""
    torch = _torch()
    n = len(stores)
    x = x.contiguous()
    m = x.shape[0]
    if outs is None:
        outs = [torch.empty((m, s.n), dtype=torch.float32, device=x.device) for s in stores]
    f, keep = _fusion(x, norm_weight, eps, gate, None)
    handles = (ctypes.c_void_p * n)(*[s.handle.value for s in stores])
    begins = (ctypes.c_int64 * n)(*([0] * n))
    rows = (ctypes.c_int64 * n)(*[o.shape[1] for o in outs])
    optrs = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
    ldos = (ctypes.c_int64 * n)(*[o.stride(0) for o in outs])
    xtype = _XTYPE.get(str(x.dtype).replace("torch.", ""))
    _lib.check(_lib.lib.clq_linear_group_fused_device(handles, begins, rows, n, x.data_ptr(), xtype, m,
                                                      ctypes.byref(f), optrs, ldos, flags,
                                                      stream if stream is not None else current_stream_handle()))
    del keep
    return outs


def linear_group(stores, x, outs=None, flags=0, stream=None):
    """One launch for up to 4 stores of one dtype and K that read the same x
    (clq_linear_group_device); returns the list of [m, rows] outputs."""
    torch = _torch()
    n = len(stores)
    if not 1 <= n <= 4:
        raise ValueError("a group holds 1 to 4 stores")
    x = x.contiguous()
    m = x.shape[0]
    if outs is None:
        outs = [torch.empty((m, s.n), dtype=torch.float32, device=x.device) for s in stores]
    handles = (ctypes.c_void_p * n)(*[s.handle.value for s in stores])
    begins = (ctypes.c_int64 * n)(*([0] * n))
    rows = (ctypes.c_int64 * n)(*[o.shape[1] for o in outs])
    optrs = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
    ldos = (ctypes.c_int64 * n)(*[o.stride(0) if o.dim() == 2 else o.shape[-1] for o in outs])
    xtype = _XTYPE.get(str(x.dtype).replace("torch.", ""))
    _lib.check(_lib.lib.clq_linear_group_device(handles, begins, rows, n, x.data_ptr(), xtype, m, optrs, ldos,
                                                flags, stream if stream is not None else current_stream_handle()))
    return outs
