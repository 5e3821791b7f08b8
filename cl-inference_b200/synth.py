"""Seeded synthetic packed weights with the value distributions of the benchmark configs.

numpy PCG64 streams, seed = 1000 * config + tensor index.  fp16 scales are
drawn in fp32 and rounded to fp16 (round to nearest even); codes are uniform
over their bit fields:
  Q8_0: d = |N(0,1)| * 0.02 / 127, int8 codes uniform in [-127, 127]
  Q4_0: d = |N(0,1)| * 0.02 / 8, 16 code bytes uniform
  Q4_K: d, dmin = |N(0,1)| * 0.01, 12 scale bytes uniform, 128 code bytes uniform
  Q6_K: ql/qh bytes uniform, int8 scales uniform in [-64, 63], d = |N(0,1)| * 0.005

quantize_q4_k / quantize_q6_k pack real-valued weights (the prefill and 70B
configurations draw them from N(0, 0.02)) into the same block formats, with
a min/max fit per sub-block (the reference has no K-format quantizer of its
own; tests/local/packed-fixtures.lisp only packs uniform sub-scales).
"""
import numpy as np

from .geometry import find_dtype


def _half_bytes(values):
    return np.asarray(values, dtype=np.float32).astype(np.float16).view(np.uint8).reshape(-1, 2)


def packed_blocks(dtype, n, k, seed):
    """Bytes of an N x K packed weight (row-major blocks) as a uint8 array."""
    dt = find_dtype(dtype)
    if k % dt.block_size:
        raise ValueError(f"K={k} is not a multiple of {dt.block_size}")
    nblocks = n * (k // dt.block_size)
    rng = np.random.Generator(np.random.PCG64(seed))
    raw = rng.integers(0, 256, size=(nblocks, dt.block_bytes), dtype=np.uint8)
    if nblocks == 0:
        return raw.reshape(-1)
    if dt.name == "q8_0":
        raw[:, 0:2] = _half_bytes(np.abs(rng.standard_normal(nblocks, dtype=np.float32)) * 0.02 / 127)
        raw[:, 2:34] = rng.integers(-127, 128, size=(nblocks, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    elif dt.name == "q4_0":
        raw[:, 0:2] = _half_bytes(np.abs(rng.standard_normal(nblocks, dtype=np.float32)) * 0.02 / 8)
    elif dt.name == "q4_k":
        raw[:, 0:2] = _half_bytes(np.abs(rng.standard_normal(nblocks, dtype=np.float32)) * 0.01)
        raw[:, 2:4] = _half_bytes(np.abs(rng.standard_normal(nblocks, dtype=np.float32)) * 0.01)
    elif dt.name == "q6_k":
        raw[:, 192:208] = rng.integers(-64, 64, size=(nblocks, 16), dtype=np.int16).astype(np.int8).view(np.uint8)
        raw[:, 208:210] = _half_bytes(np.abs(rng.standard_normal(nblocks, dtype=np.float32)) * 0.005)
    return raw.reshape(-1)


def activations(m, k, seed):
    """fp32 N(0,1) activations [m, k]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal((m, k), dtype=np.float32)


def _fp16(v):
    return np.asarray(v, np.float32).astype(np.float16)


def quantize_q4_k(w):
    """Q4_K bytes of an [n, k] float weight (k a multiple of 256).

    Per 32-element sub-block j: the range [min(x, 0), max(x)] splits into 15
    steps, scale_j = (max - min') / 15 and offset_j = -min'; the superblock's
    fp16 d and dmin are the largest scale and offset over 63, the 6-bit
    sub-scales sc_j = rint(scale_j / d) and m_j = rint(offset_j / dmin), and the
    codes q = rint((x + dmin m_j) / (d sc_j)) in [0, 15], so that x ~ d sc_j q -
    dmin m_j, the element formula of quant/packed.lisp:89-100."""
    w = np.asarray(w, np.float32)
    n, k = w.shape
    if k % 256:
        raise ValueError(f"K={k} is not a multiple of 256")
    x = w.reshape(-1, 8, 32)
    lo = np.minimum(x.min(axis=2), 0.0).astype(np.float32)
    hi = np.maximum(x.max(axis=2), 0.0).astype(np.float32)
    scale = ((hi - lo) / np.float32(15)).astype(np.float32)
    off = (-lo).astype(np.float32)
    d = _fp16(scale.max(axis=1) / np.float32(63))
    dmin = _fp16(off.max(axis=1) / np.float32(63))
    d32, dm32 = d.astype(np.float32)[:, None], dmin.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32 > 0, np.rint(scale / d32), 0).clip(0, 63).astype(np.int32)
        m = np.where(dm32 > 0, np.rint(off / dm32), 0).clip(0, 63).astype(np.int32)
        step = (d32 * sc.astype(np.float32)).astype(np.float32)[:, :, None]
        base = (dm32 * m.astype(np.float32)).astype(np.float32)[:, :, None]
        q = np.where(step > 0, np.rint((x + base) / step), 0).clip(0, 15).astype(np.uint8)
    nb = x.shape[0]
    out = np.zeros((nb, 144), np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
    # 6-bit sc/m of sub-blocks 0..3 in bytes 0..7, those of 4..7 split into
    # low nibbles (bytes 8..11) and top bits (bits 6..7 of bytes 0..7)
    out[:, 4:8] = (sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)).astype(np.uint8)
    out[:, 8:12] = (m[:, 0:4] | ((m[:, 4:8] >> 4) << 6)).astype(np.uint8)
    out[:, 12:16] = ((sc[:, 4:8] & 15) | ((m[:, 4:8] & 15) << 4)).astype(np.uint8)
    # codes: byte 32 p + l holds sub-block 2p (low nibble) and 2p + 1 (high)
    out[:, 16:144] = (q[:, 0::2, :] | (q[:, 1::2, :] << 4)).reshape(nb, 128)
    return out.reshape(-1)


def quantize_q6_k(w):
    """Q6_K bytes of an [n, k] float weight (k a multiple of 256).

    Per 16-element group j: scale_j = max|x| / 31; the superblock's fp16 d is
    the largest scale over 127, the int8 sub-scale sc_j = rint(scale_j / d),
    and the 6-bit codes q = rint(x / (d sc_j)) + 32 in [0, 63], so that
    x ~ d sc_j (q - 32), the element formula of quant/packed.lisp:101-108."""
    w = np.asarray(w, np.float32)
    n, k = w.shape
    if k % 256:
        raise ValueError(f"K={k} is not a multiple of 256")
    x = w.reshape(-1, 16, 16)
    scale = (np.abs(x).max(axis=2) / np.float32(31)).astype(np.float32)
    d = _fp16(scale.max(axis=1) / np.float32(127))
    d32 = d.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32 > 0, np.rint(scale / d32), 0).clip(-128, 127).astype(np.int32)
        step = (d32 * sc.astype(np.float32)).astype(np.float32)[:, :, None]
        q = (np.where(step != 0, np.rint(x / step), 0) + 32).clip(0, 63).astype(np.uint8)
    nb = x.shape[0]
    q = q.reshape(nb, 2, 4, 32)  # [block][h][g][l]: element 128 h + 32 g + l
    out = np.zeros((nb, 210), np.uint8)
    ql = out[:, 0:128].reshape(nb, 2, 2, 32)     # [h][g % 2][l], nibble g // 2
    ql[...] = (q[:, :, 0:2, :] & 15) | ((q[:, :, 2:4, :] & 15) << 4)
    qh = out[:, 128:192].reshape(nb, 2, 32)      # [h][l], bits 2 g
    qh[...] = (q[:, :, 0, :] >> 4) | ((q[:, :, 1, :] >> 4) << 2) | ((q[:, :, 2, :] >> 4) << 4) | ((q[:, :, 3, :] >> 4) << 6)
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return out.reshape(-1)


def normal_weight(n, k, seed, std=0.02):
    """An [n, k] float32 weight drawn from N(0, std^2)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.standard_normal((n, k), dtype=np.float32) * np.float32(std)).astype(np.float32)


# ---- the same quantizers on torch tensors (device-side weights for the
# benchmark's large configurations; the bytes equal the numpy versions') ----

def _fp16_t(torch, v):
    return v.to(torch.float32).to(torch.float16)


def quantize_q4_k_torch(w):
    """quantize_q4_k for a torch float32 [n, k] tensor (any device): uint8 bytes."""
    import torch
    n, k = w.shape
    x = w.to(torch.float32).reshape(-1, 8, 32)
    lo = torch.clamp(x.amin(dim=2), max=0.0)
    hi = torch.clamp(x.amax(dim=2), min=0.0)
    scale = (hi - lo) / 15.0
    off = -lo
    d = _fp16_t(torch, scale.amax(dim=1) / 63.0)
    dmin = _fp16_t(torch, off.amax(dim=1) / 63.0)
    d32, dm32 = d.float()[:, None], dmin.float()[:, None]
    zero = torch.zeros((), device=w.device)
    sc = torch.where(d32 > 0, torch.round(scale / torch.where(d32 > 0, d32, 1.0)), zero).clamp(0, 63).to(torch.int32)
    m = torch.where(dm32 > 0, torch.round(off / torch.where(dm32 > 0, dm32, 1.0)), zero).clamp(0, 63).to(torch.int32)
    step = (d32 * sc.float())[:, :, None]
    base = (dm32 * m.float())[:, :, None]
    q = torch.where(step > 0, torch.round((x + base) / torch.where(step > 0, step, 1.0)), zero).clamp(0, 15)
    q = q.to(torch.uint8)
    nb = x.shape[0]
    out = torch.zeros((nb, 144), dtype=torch.uint8, device=w.device)
    out[:, 0:2] = d.view(torch.uint8).reshape(-1, 2)
    out[:, 2:4] = dmin.view(torch.uint8).reshape(-1, 2)
    out[:, 4:8] = (sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)).to(torch.uint8)
    out[:, 8:12] = (m[:, 0:4] | ((m[:, 4:8] >> 4) << 6)).to(torch.uint8)
    out[:, 12:16] = ((sc[:, 4:8] & 15) | ((m[:, 4:8] & 15) << 4)).to(torch.uint8)
    out[:, 16:144] = (q[:, 0::2, :] | (q[:, 1::2, :] << 4)).reshape(nb, 128)
    return out.reshape(-1)


def quantize_q6_k_torch(w):
    """quantize_q6_k for a torch float32 [n, k] tensor (any device): uint8 bytes."""
    import torch
    n, k = w.shape
    x = w.to(torch.float32).reshape(-1, 16, 16)
    scale = x.abs().amax(dim=2) / 31.0
    d = _fp16_t(torch, scale.amax(dim=1) / 127.0)
    d32 = d.float()[:, None]
    zero = torch.zeros((), device=w.device)
    sc = torch.where(d32 > 0, torch.round(scale / torch.where(d32 > 0, d32, 1.0)), zero).clamp(-128, 127)
    sc = sc.to(torch.int32)
    step = (d32 * sc.float())[:, :, None]
    q = (torch.where(step != 0, torch.round(x / torch.where(step != 0, step, 1.0)), zero) + 32).clamp(0, 63)
    q = q.to(torch.uint8)
    nb = x.shape[0]
    q = q.reshape(nb, 2, 4, 32)
    out = torch.zeros((nb, 210), dtype=torch.uint8, device=w.device)
    out[:, 0:128] = ((q[:, :, 0:2, :] & 15) | ((q[:, :, 2:4, :] & 15) << 4)).reshape(nb, 128)
    out[:, 128:192] = ((q[:, :, 0, :] >> 4) | ((q[:, :, 1, :] >> 4) << 2) | ((q[:, :, 2, :] >> 4) << 4)
                       | ((q[:, :, 3, :] >> 4) << 6)).reshape(nb, 64)
    out[:, 192:208] = sc.to(torch.int8).view(torch.uint8)
    out[:, 208:210] = d.view(torch.uint8).reshape(-1, 2)
    return out.reshape(-1)
