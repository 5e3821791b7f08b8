"""The Q4_K / Q6_K quantizers of synth.py (no GPU needed).

They make the N(0, 0.02) weights of the prefill and 70B configurations.  Their
bytes must decode the same through the oracle (the reference's element
formulas, quant/packed.lisp:89-108) and through llama.cpp's Python decoder
(gguf 0.19.0, gguf.quants.dequantize); the decoded values must stay within
half a quantization step of the input (plus the fp16 rounding of the
scales), and the numpy and torch forms must give the same bytes.
"""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as T  # noqa: E402
import gguf.quants as gq  # noqa: E402

TYPES = {"q4_k": T.Q4_K, "q6_k": T.Q6_K}


def weights():
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((12, 512)) * 0.02).astype(np.float32)
    w[0] = 0.0                           # all zeros
    w[1] = 0.013                         # constant, positive
    w[2] = -np.abs(w[2])                 # negative only
    w[3, :256] *= 1e4                    # one large superblock
    w[4, 7] = 3.0                        # an outlier
    w[5] = np.float32(1e-30) * np.sign(w[5])  # tiny values (fp16 scales underflow)
    return w


@pytest.mark.parametrize("dtype", ["q4_k", "q6_k"])
def test_bytes_decode_the_same_through_oracle_and_gguf(synth, oracle, dtype):
    w = weights()
    b = getattr(synth, "quantize_" + dtype)(w)
    assert b.dtype == np.uint8 and b.size == w.size // 256 * {"q4_k": 144, "q6_k": 210}[dtype]
    ours = oracle.dequantize(dtype, b)
    theirs = gq.dequantize(b, TYPES[dtype]).astype(np.float32).ravel()
    assert np.array_equal(ours.view(np.uint32), theirs.view(np.uint32))
    assert np.all(np.isfinite(ours))


@pytest.mark.parametrize("dtype,rel", [("q4_k", 0.10), ("q6_k", 0.03)])
def test_error_of_normal_weights(synth, oracle, dtype, rel):
    w = synth.normal_weight(64, 1024, seed=5)
    deq = oracle.dequantize(dtype, getattr(synth, "quantize_" + dtype)(w)).reshape(w.shape)
    err = np.sqrt(np.mean((deq - w) ** 2)) / np.sqrt(np.mean(w ** 2))
    assert err < rel, err


def test_q4_k_elements_within_half_a_step(synth, oracle):
    w = weights()
    b = synth.quantize_q4_k(w).reshape(-1, 144)
    deq = oracle.dequantize("q4_k", b.reshape(-1)).reshape(-1, 8, 32)
    x = w.reshape(-1, 8, 32)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    # the largest sub-block step is d * 63; every element is within half of
    # it plus what the 6-bit rounding of scale and offset can add (a step)
    bound = (d * 63.0)[:, None, None] * 1.5 + 1e-6 * np.abs(x).max(axis=(1, 2), keepdims=True)
    assert np.all(np.abs(deq - x) <= bound + 1e-30)


@pytest.mark.parametrize("dtype", ["q4_k", "q6_k"])
def test_numpy_and_torch_give_the_same_bytes(synth, dtype):
    torch = pytest.importorskip("torch")
    w = weights()
    a = getattr(synth, "quantize_" + dtype)(w)
    t = getattr(synth, "quantize_" + dtype + "_torch")(torch.from_numpy(w)).numpy()
    assert np.array_equal(a, t)
