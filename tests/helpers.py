"""Tolerances and fixture builders shared by the tests."""
import numpy as np

# tests/local/packed.lisp:5-12: |out - sum| <= 1e-5 + 1e-5 * sum|x*w| against fp64
ELEMENT_ABS, ELEMENT_REL = 1e-5, 1e-5
# the gate for linear outputs: max over activation rows of ||y - y64|| / ||y64||
NORM_REL = 1e-3


def element_bound_ok(out, ref, mag, abs_tol=ELEMENT_ABS, rel_tol=ELEMENT_REL):
    return np.all(np.abs(out.astype(np.float64) - ref) <= abs_tol + rel_tol * mag)


def max_row_relative_error(out, ref):
    out = out.astype(np.float64)
    num = np.linalg.norm(out - ref, axis=-1)
    den = np.maximum(np.linalg.norm(ref, axis=-1), 1e-300)
    return float(np.max(num / den))


def q8_activations(rows, columns):
    """tests/local/quant.lisp:19-22: 0.1 * (((5r + 3c) mod 11) - 5)."""
    r = np.arange(rows)[:, None]
    c = np.arange(columns)[None, :]
    return (np.float32(0.1) * (((5 * r + 3 * c) % 11) - 5).astype(np.float32)).astype(np.float32)


def weight_values(name, count):
    """tests/local/fixtures.lisp:32-39 (non-norm tensors): 0.5 * sin(seed + 1.3 i)."""
    seed = sum(ord(ch) for ch in name)
    i = np.arange(count, dtype=np.float64)
    return (0.5 * np.sin(seed + 1.3 * i)).astype(np.float32)


def q8_0_octets(values):
    """ggml-style Q8_0 packing of tests/local/fixtures.lisp:52-65,76-80."""
    values = np.asarray(values, np.float32).reshape(-1, 32)
    out = np.zeros((values.shape[0], 34), np.uint8)
    for b, block in enumerate(values):
        scale = np.float32(np.max(np.abs(block)) / np.float32(127))
        stored = np.float16(scale)
        out[b, 0:2] = np.array([stored], np.float16).view(np.uint8)
        if stored == 0:
            q = np.zeros(32, np.int64)
        else:
            q = np.rint(block.astype(np.float64) / np.float64(scale)).astype(np.int64)
        out[b, 2:] = q.astype(np.int8).view(np.uint8)
    return out.reshape(-1)
