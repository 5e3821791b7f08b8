"""The CPU oracle pinned against the reference's golden vectors (CPU only).

Mirrors tests/local/packed.lisp:14-33 (exact dequantization against the
llama.cpp blocks of tests/local/quant-golden.lisp) and the Q8_0 golden of
tests/mlx-gguf/kernels.lisp:9-21, plus the error paths of
tests/local/packed.lisp:48-52.
"""
import numpy as np
import pytest

DTYPES = ["q8_0", "q4_0", "q4_k", "q6_k"]


@pytest.mark.parametrize("dtype", DTYPES)
def test_oracle_matches_golden_bit_for_bit(oracle, golden, dtype):
    g = golden[dtype]
    got = oracle.dequantize(dtype, g["bytes"])
    # bit patterns, so -0.0 and 0.0 are told apart
    assert np.array_equal(got.view(np.uint32), g["values"].view(np.uint32))


@pytest.mark.parametrize("dtype", DTYPES)
def test_oracle_element_walk_matches_golden(oracle, golden, dtype):
    import ctypes
    g = golden[dtype]
    e, b = oracle.geometry(dtype)
    data = g["bytes"]
    for blk in range(5):
        for i in range(0, e, 7):
            out = ctypes.c_float()
            rc = oracle.lib.clqo_element(oracle.GGML[dtype], data[blk * b:].ctypes.data, i, ctypes.byref(out))
            assert rc == 0
            assert np.float32(out.value).view(np.uint32) == g["values"][blk * e + i].view(np.uint32)


@pytest.mark.parametrize("dtype", DTYPES)
def test_oracle_rejects_nonfinite_scales(oracle, golden, dtype):
    g = golden[dtype]
    for offset in g["bad_offsets"]:
        bad = g["bytes"].copy()
        bad[offset] = 0x7C  # exponent 31 in the scale's high byte
        with pytest.raises(oracle.OracleError) as err:
            oracle.dequantize(dtype, bad)
        assert err.value.code == oracle.ERR_NONFINITE


def test_block_scale_matches_ieee_half(oracle):
    # quant/q8-0.lisp:89-96 over every finite half bit pattern
    for bits in range(0, 1 << 16, 7):
        lo, hi = bits & 255, bits >> 8
        if (bits >> 10) & 31 == 31:
            with pytest.raises(oracle.OracleError):
                oracle.block_scale(lo, hi)
            continue
        expect = np.array([bits], np.uint16).view(np.float16).astype(np.float32)[0]
        assert oracle.block_scale(lo, hi).view(np.uint32) == expect.view(np.uint32)


@pytest.mark.parametrize("dtype", DTYPES)
def test_oracle_agrees_with_gguf_decoder_on_synthetic_blocks(oracle, synth, dtype):
    gq = pytest.importorskip("gguf.quants")
    from gguf import GGMLQuantizationType as T
    qtype = {"q4_0": T.Q4_0, "q8_0": T.Q8_0, "q4_k": T.Q4_K, "q6_k": T.Q6_K}[dtype]
    e, _ = oracle.geometry(dtype)
    data = synth.packed_blocks(dtype, 8, 4 * e, seed=11)
    ours = oracle.dequantize(dtype, data)
    theirs = gq.dequantize(data, qtype).astype(np.float32).ravel()
    assert np.array_equal(ours.view(np.uint32), theirs.view(np.uint32))


@pytest.mark.parametrize("dtype", DTYPES)
def test_oracle_matmul_against_numpy(oracle, synth, dtype):
    e, _ = oracle.geometry(dtype)
    n, k = 37, 3 * e
    data = synth.packed_blocks(dtype, n, k, seed=5)
    w = oracle.dequantize(dtype, data).reshape(n, k).astype(np.float64)
    for m in (1, 3, 5, 9):
        x = synth.activations(m, k, seed=m)
        ref, mag = oracle.matmul_f64(dtype, x, data, n)
        np.testing.assert_allclose(ref, x.astype(np.float64) @ w.T, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(mag, np.abs(x.astype(np.float64)[:, None, :] * w[None]).sum(-1), rtol=1e-12)
        f32 = oracle.matmul_f32(dtype, x, data, n)
        # the reference's tested bound for the native kernels (tests/local/packed.lisp:5-12)
        assert np.all(np.abs(f32 - ref) <= 1e-5 + 1e-5 * mag)


def test_oracle_gather_matches_rows(oracle, synth):
    data = synth.packed_blocks("q4_k", 6, 512, seed=3)
    rows = oracle.dequantize("q4_k", data).reshape(6, 512)
    ids = np.array([4, 1, 4, 0], np.int32)
    assert np.array_equal(oracle.gather("q4_k", data, 6, 512, ids), rows[ids])


@pytest.mark.parametrize("dtype", DTYPES)
def test_block_decoder_equals_element_walk(oracle, synth, dtype):
    """clqo_dequantize's per-block decoder against packed-element one element at a time."""
    import ctypes
    e, b = oracle.geometry(dtype)
    data = synth.packed_blocks(dtype, 4, 2 * e, seed=17)
    fast = oracle.dequantize(dtype, data)
    for i in range(0, fast.size, 3):
        out = ctypes.c_float()
        oracle.lib.clqo_element(oracle.GGML[dtype], data[(i // e) * b:].ctypes.data, i % e, ctypes.byref(out))
        assert np.float32(out.value).view(np.uint32) == fast[i].view(np.uint32)
