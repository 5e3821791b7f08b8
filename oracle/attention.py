"""CPU restatement of the reference's KV cache codec, RoPE and attention.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker of the device
cache, RoPE and attention kernels; never imported by the product.

Each function follows the cl-inference lines it cites.  Element arithmetic is
float32 where the reference's is single-float (the Q8 codec, the RoPE
rotation), float64 where an exact reference value is wanted (attention); the
softmax is the standard max-subtracted form (cl-tensor's ct:softmax, which is
not vendored with the reference).
"""
import math

import numpy as np

Q8_GROUP = 32  # local/kv-cache.lisp:20
F32_MAX = float(np.finfo(np.float32).max)
F32_MIN_NORMAL = float(np.finfo(np.float32).tiny)


class NonFinite(ValueError):
    """A non-finite key or value offered to the Q8 codec (local/kv-cache.lisp:49)."""


def q8_store(rows):
    """store-q8-rows (local/kv-cache.lisp:37-60): ROWS (count, heads, dim)
    float32 -> int8 codes of the same shape and float32 scales
    (count, heads, ceil(dim / 32)).  Per group of 32: peak |value|, scale =
    single(max(least-positive-normalized, peak / 127)) in double (1 for a zero
    peak), code = clamp(round-half-even(value / scale), -127, 127) with the
    division in single precision."""
    rows = np.asarray(rows, dtype=np.float32)
    count, heads, dim = rows.shape
    groups = -(-dim // Q8_GROUP)
    codes = np.zeros((count, heads, dim), dtype=np.int8)
    scales = np.ones((count, heads, groups), dtype=np.float32)
    for r in range(count):
        for h in range(heads):
            for g in range(groups):
                seg = rows[r, h, g * Q8_GROUP:(g + 1) * Q8_GROUP]
                if not np.all(np.isfinite(seg)):
                    raise NonFinite("Non-finite key or value")
                peak = float(np.max(np.abs(seg))) if seg.size else 0.0
                scale = np.float32(1.0) if peak == 0.0 else np.float32(max(F32_MIN_NORMAL, peak / 127.0))
                scales[r, h, g] = scale
                q = np.rint(seg / scale)  # float32 / float32 -> float32; rint rounds half to even
                codes[r, h, g * Q8_GROUP:g * Q8_GROUP + seg.size] = np.clip(q, -127, 127).astype(np.int8)
    return codes, scales


def q8_prefix(codes, scales):
    """q8-prefix (local/kv-cache.lisp:62-78): codes (end, heads, dim), scales
    (end, heads, groups) -> float32 values: code * scale in single precision
    when scale <= FLT_MAX / 127, else the double product clamped to the finite
    range."""
    codes = np.asarray(codes, dtype=np.int8)
    scales = np.asarray(scales, dtype=np.float32)
    dim = codes.shape[2]
    s = np.repeat(scales, Q8_GROUP, axis=2)[:, :, :dim]
    with np.errstate(over="ignore"):
        out = codes.astype(np.float32) * s
    limit = F32_MAX / 127.0
    big = s.astype(np.float64) > limit
    if np.any(big):
        wide = np.clip(codes.astype(np.float64) * s.astype(np.float64), -F32_MAX, F32_MAX).astype(np.float32)
        out = np.where(big, wide, out)
    return out


def rope_tables(start, count, rope_dims, theta, factors=None):
    """rope-tables (local/blocks.lisp:172-184): cos and sin (count, rope_dims/2)
    float32, frequency i = theta^(-2i / rope_dims) / factors[i] and angle
    (start + pos) * frequency in double, rounded to single at the end."""
    half = rope_dims // 2
    cos = np.zeros((count, half), dtype=np.float32)
    sin = np.zeros((count, half), dtype=np.float32)
    for i in range(half):
        frequency = float(theta) ** ((-2.0 * i) / rope_dims)
        if factors is not None:
            frequency /= float(np.float32(factors[i]))
        for pos in range(count):
            angle = (start + pos) * frequency
            cos[pos, i] = np.float32(math.cos(angle))
            sin[pos, i] = np.float32(math.sin(angle))
    return cos, sin


def apply_rope(x, cos, sin, pairing, rope_dims):
    """apply-rope (local/blocks.lisp:190-214) on X (count, heads, head_dim)
    float32: pairs (2i, 2i+1) (adjacent) or (i, i + half) (neox) rotated with
    x0 cos - x1 sin, x0 sin + x1 cos, each product and sum in single precision;
    the dimensions past rope_dims pass through."""
    x = np.array(x, dtype=np.float32, copy=True)
    half = rope_dims // 2
    c = cos[:, None, :]
    s = sin[:, None, :]
    if pairing == "adjacent":
        x0, x1 = x[:, :, 0:rope_dims:2].copy(), x[:, :, 1:rope_dims:2].copy()
        x[:, :, 0:rope_dims:2] = x0 * c - x1 * s
        x[:, :, 1:rope_dims:2] = x0 * s + x1 * c
    elif pairing == "neox":
        x0, x1 = x[:, :, :half].copy(), x[:, :, half:rope_dims].copy()
        x[:, :, :half] = x0 * c - x1 * s
        x[:, :, half:rope_dims] = x0 * s + x1 * c
    else:
        raise ValueError(pairing)
    return x


def causal_mask(count, key_count, query_start, key_start):
    """causal-mask (local/blocks.lisp:282-292) without a window: (count,
    key_count) booleans, True where the key's position is not after the
    query's; None when nothing is masked."""
    q = query_start + np.arange(count)[:, None]
    k = key_start + np.arange(key_count)[None, :]
    mask = k <= q
    return None if mask.all() else mask


def attend_f64(q, keys, values, mask, n_heads, n_kv_heads):
    """attend (local/blocks.lisp:308-325) in float64: per head h, KV head
    h // (n_heads / n_kv_heads), scores (q . k) / sqrt(head_dim), masked
    scores -1e30, softmax over keys, weighted sum of values; heads
    concatenated along the last axis -> (count, n_heads * head_dim)."""
    q = np.asarray(q, dtype=np.float64)
    keys = np.asarray(keys, dtype=np.float64)
    values = np.asarray(values, dtype=np.float64)
    count, _, head_dim = q.shape
    group = n_heads // n_kv_heads
    scale = float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))
    out = np.zeros((count, n_heads * head_dim))
    for h in range(n_heads):
        kv = h // group
        scores = q[:, h, :] @ keys[:, kv, :].T * scale
        if mask is not None:
            scores = np.where(mask, scores, -1e30)
        scores = scores - scores.max(axis=1, keepdims=True)
        p = np.exp(scores)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h * head_dim:(h + 1) * head_dim] = p @ values[:, kv, :]
    return out
