"""Seeded synthetic packed weights with the value distributions of the benchmark configs.

numpy PCG64 streams, seed = 1000 * config + tensor index.  fp16 scales are
drawn in fp32 and rounded to fp16 (round to nearest even); codes are uniform
over their bit fields:
  Q8_0: d = |N(0,1)| * 0.02 / 127, int8 codes uniform in [-127, 127]
  Q4_0: d = |N(0,1)| * 0.02 / 8, 16 code bytes uniform
  Q4_K: d, dmin = |N(0,1)| * 0.01, 12 scale bytes uniform, 128 code bytes uniform
  Q6_K: ql/qh bytes uniform, int8 scales uniform in [-64, 63], d = |N(0,1)| * 0.005
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
