"""KV cache, RoPE and grouped-query attention on the device (clq_kv_cache_*,
clq_rope_device, clq_attend_device).

The layer work between the projections of local/blocks.lisp:327-353:
  KVCache(n_ctx, layers, kv_heads, head_dim, cache_type="f32"|"q8")
      make-kv-cache (local/kv-cache.lisp:17-19), every layer's keys and values
      in device memory; update(layer, k, v, start) is the store half of
      kv-cache-update (:92-110) and prefix(layer, end) its returned prefix
      (the f32 slice, or q8-prefix :62-78).
  rope(x, start, theta, rope_dims=None, pairing="adjacent", factors=None)
      apply-rope with rope-tables (local/blocks.lisp:172-214), in place.
  attend(q, cache, layer, end, query_start)
      attend with causal-mask (:282-325) over the cached prefix.
  llama3_rope_factors(dims, theta, scaling)
      the per-frequency divisors of llama3-rope-factors (:230-252).

Tensors are torch CUDA f32 tensors: rows (positions, heads, head_dim) with a
unit last stride.  Errors raise ClqError: CLQ_ERR_CONTEXT past the context
(the reference's context-overflow), CLQ_ERR_NONFINITE_VALUE for a non-finite
value stored into a Q8 cache (reported by update(check=True) or status()).
"""
import ctypes
import math

from . import _lib
from .store import current_stream_handle

CACHE_TYPES = {"f32": 0, "q8": 1}
PAIRINGS = {"adjacent": 0, "neox": 1}


def _torch():
    import torch
    return torch


def _rows(t, what):
    torch = _torch()
    if t.dtype != torch.float32 or not t.is_cuda or t.dim() != 3 or t.stride(2) != 1:
        raise ValueError(f"{what}: a CUDA float32 tensor (positions, heads, head_dim) with unit last stride")
    return t


class KVCache:
    def __init__(self, n_ctx, layers, kv_heads, head_dim, cache_type="f32"):
        if cache_type not in CACHE_TYPES:
            raise _lib.ClqError(1, f"unknown cache type {cache_type!r} (f32 or q8)")
        handle = ctypes.c_void_p()
        _lib.check(_lib.lib.clq_kv_cache_create(n_ctx, layers, kv_heads, head_dim, CACHE_TYPES[cache_type],
                                                ctypes.byref(handle)))
        self._handle = handle
        self.n_ctx, self.layers, self.kv_heads, self.head_dim = n_ctx, layers, kv_heads, head_dim
        self.cache_type = cache_type

    @property
    def handle(self):
        if self._handle is None:
            raise ValueError("KV cache is closed")
        return self._handle

    def update(self, layer, k, v, start, check=False, stream=None):
        """Store K and V rows (count, kv_heads, head_dim) at positions start..;
        with CHECK, wait and raise for a non-finite value into a Q8 cache."""
        k, v = _rows(k, "k"), _rows(v, "v")
        if k.shape != v.shape or k.shape[1:] != (self.kv_heads, self.head_dim):
            raise ValueError(f"k {tuple(k.shape)} / v {tuple(v.shape)} rows for {self.kv_heads} heads of {self.head_dim}")
        if k.stride() != v.stride():
            raise ValueError("k and v rows must share their strides")
        _lib.check(_lib.lib.clq_kv_cache_update(self.handle, layer, k.data_ptr(), v.data_ptr(), k.shape[0], k.stride(0),
                                                k.stride(1), start,
                                                stream if stream is not None else current_stream_handle()))
        if check:
            self.raise_status()

    def status(self):
        st = ctypes.c_int()
        _lib.check(_lib.lib.clq_kv_cache_status(self.handle, ctypes.byref(st)))
        return st.value

    def raise_status(self):
        st = self.status()
        if st:
            raise _lib.ClqError(st, "Non-finite key or value")

    def prefix(self, layer, end, stream=None):
        """LAYER's first END positions as f32 (keys, values), each (end, kv_heads, head_dim)."""
        torch = _torch()
        keys = torch.empty((end, self.kv_heads, self.head_dim), dtype=torch.float32, device="cuda")
        values = torch.empty_like(keys)
        _lib.check(_lib.lib.clq_kv_cache_read(self.handle, layer, end, keys.data_ptr(), values.data_ptr(),
                                              stream if stream is not None else current_stream_handle()))
        return keys, values

    def close(self):
        if self._handle is not None:
            _lib.lib.clq_kv_cache_destroy(self._handle)
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


def rope(x, start, theta, rope_dims=None, pairing="adjacent", factors=None, stream=None):
    """Rotate the first ROPE_DIMS of each head of X (positions, heads, head_dim) in place."""
    x = _rows(x, "x")
    if pairing not in PAIRINGS:
        raise ValueError(f"unknown pairing {pairing!r}")
    rope_dims = x.shape[2] if rope_dims is None else rope_dims
    fptr = None
    if factors is not None:
        torch = _torch()
        if factors.dtype != torch.float32 or not factors.is_cuda or factors.numel() < rope_dims // 2:
            raise ValueError("factors: a CUDA float32 tensor of rope_dims / 2 values")
        fptr = factors.contiguous().data_ptr()
    _lib.check(_lib.lib.clq_rope_device(x.data_ptr(), x.shape[0], x.shape[1], x.shape[2], x.stride(0), x.stride(1),
                                        rope_dims, start, float(theta), fptr, PAIRINGS[pairing],
                                        stream if stream is not None else current_stream_handle()))
    return x


def attend(q, cache, layer, end, query_start, out=None, stream=None):
    """Attention of Q (count, n_heads, head_dim) over LAYER's cached positions
    [0, END); row t sits at position QUERY_START + t.  Returns (count, n_heads * head_dim)."""
    torch = _torch()
    q = _rows(q, "q")
    if q.stride(1) != q.shape[2]:
        raise ValueError("q: heads must be contiguous within a position")
    count, heads, hd = q.shape
    if out is None:
        out = torch.empty((count, heads * hd), dtype=torch.float32, device=q.device)
    _lib.check(_lib.lib.clq_attend_device(q.data_ptr(), count, heads, q.stride(0), cache.handle, layer, end,
                                          query_start, out.data_ptr(), out.stride(0),
                                          stream if stream is not None else current_stream_handle()))
    return out


def llama3_rope_factors(dims, theta, scaling):
    """Per-frequency divisors for Llama 3 RoPE scaling (llama3-rope-factors,
    local/blocks.lisp:230-252), as f32 values in a list; None for "default"."""
    mode = scaling.get("rope_type", scaling.get("type"))
    if mode == "default":
        return None
    if mode != "llama3":
        raise ValueError(f"Unsupported RoPE scaling {mode!r}")
    factor, low = scaling.get("factor"), scaling.get("low_freq_factor")
    high, context = scaling.get("high_freq_factor"), scaling.get("original_max_position_embeddings")
    if not (isinstance(factor, (int, float)) and factor >= 1 and isinstance(low, (int, float)) and low > 0
            and isinstance(high, (int, float)) and high > low and isinstance(context, int) and context > 0):
        raise ValueError("Invalid Llama 3 RoPE scaling parameters")
    import numpy as np
    out = []
    for i in range(dims // 2):
        frequency = float(theta) ** (-2.0 * i / dims)
        wavelength = 2 * math.pi / frequency
        smooth = (context / wavelength - low) / (high - low)
        if wavelength < context / high:
            multiplier = 1.0
        elif wavelength > context / low:
            multiplier = 1.0 / factor
        else:
            multiplier = (1 - smooth) / factor + smooth
        out.append(float(np.float32(1.0 / multiplier)))
    return out
