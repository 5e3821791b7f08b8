"""CUDA kernels of libclq against the CPU oracle (needs a B200).

Mirrors tests/local/packed.lisp (dequantization, views, matmul bound),
tests/local/quant.lisp (Q8_0 products) and tests/mlx-gguf/kernels.lisp
(GPU projections, gathers, load-time scale checks), then checks every
benchmark configuration's shapes against the fp64 oracle.
"""
import ctypes

import numpy as np
import pytest

from helpers import (NORM_REL, element_bound_ok, max_row_relative_error, q8_0_octets,
                     q8_activations, weight_values)

pytestmark = pytest.mark.gpu
DTYPES = ["q8_0", "q4_0", "q4_k", "q6_k"]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---- dequantize / gather: bit-exact --------------------------------------


@pytest.mark.parametrize("dtype", DTYPES)
def test_dequantize_matches_golden_bit_for_bit(cuda, clq, golden, dtype):
    g = golden[dtype]
    k = g["elements"]
    weight = clq.make_tensor_view(clq.make_packed_storage(dtype, g["bytes"]), (5, k))
    decoded = clq.dequantize(weight)
    assert np.array_equal(bits(decoded.ravel()), bits(g["values"]))
    flipped = clq.astype(clq.transpose(weight), "f32")
    assert np.array_equal(bits(flipped), bits(decoded.T))
    taken = clq.dequantize(clq.take(weight, [4, 1, 4]))
    assert np.array_equal(bits(taken), bits(decoded[[4, 1, 4]]))
    assert np.array_equal(bits(clq.take_dequantized(weight, [4, 1, 4])), bits(decoded[[4, 1, 4]]))


@pytest.mark.parametrize("dtype", DTYPES)
def test_device_dequantize_and_gather_match_oracle(cuda, clq, synth, oracle, dtype):
    torch = cuda
    e = clq.DTYPES[dtype].block_size
    n, k = 67, 8 * e
    data = synth.packed_blocks(dtype, n, k, seed=21)
    expect = oracle.dequantize(dtype, data).reshape(n, k)
    store = clq.Store(dtype, n, k, data)
    got = store.dequantize().cpu().numpy()
    assert np.array_equal(bits(got), bits(expect))
    part = store.dequantize(row_begin=5, rows=9, transposed=True).cpu().numpy()
    assert np.array_equal(bits(part), bits(expect[5:14].T))
    ids = torch.tensor([66, 0, 3, 3, 17], dtype=torch.int32, device="cuda")
    gathered = store.gather(ids).cpu().numpy()
    assert np.array_equal(bits(gathered), bits(oracle.gather(dtype, data, n, k, ids.cpu().numpy())))
    store.close()


# ---- products on the reference's own fixtures ------------------------------


@pytest.mark.parametrize("dtype", DTYPES)
def test_packed_matmul_within_reference_bound(cuda, clq, oracle, golden, dtype):
    """tests/local/packed.lisp:53-60: M in {1,3,5,9}, offset views, zero rows."""
    g = golden[dtype]
    k = g["elements"]
    storage = clq.make_packed_storage(dtype, g["bytes"])
    weight = clq.make_tensor_view(storage, (5, k))
    assert clq.linear(np.zeros((0, k), np.float32), weight).shape == (0, 5)
    for m in (1, 3, 5, 9):
        x = q8_activations(m, k)
        out = clq.matmul(x, clq.transpose(weight))
        ref, mag = oracle.matmul_f64(dtype, x, g["bytes"], 5)
        assert element_bound_ok(out, ref, mag), (dtype, m)
    if dtype != "q8_0":
        x = q8_activations(4, k)[1:3]
        view = clq.make_tensor_view(storage, (3, k), offset=k)
        out = clq.matmul(x, clq.transpose(view))
        ref, mag = oracle.matmul_f64(dtype, x, g["bytes"][g["block_bytes"]:], 3)
        assert element_bound_ok(out, ref, mag)


def test_q8_0_matmul_matches_dequantized_values(cuda, clq, oracle):
    """tests/local/quant.lisp:38-49: 40 x 96 Q8_0 weight, M in {1,3,6,9}, 1e-3."""
    data = q8_0_octets(weight_values("w40.96", 40 * 96))
    weight = clq.make_tensor_view(clq.make_q8_0_storage(data), (40, 96))
    for m in (1, 3, 6, 9):
        x = q8_activations(m, 96)
        out = clq.linear(x, weight)
        ref, _ = oracle.matmul_f64("q8_0", x, data, 40)
        assert np.max(np.abs(out - ref)) <= 1e-3


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("blocks", [1, 5])
def test_gpu_projections_match_f64(cuda, clq, golden, dtype, blocks):
    """tests/mlx-gguf/kernels.lisp:26-58: rows x (elements*blocks) weights,
    batches {1,3,9} of x = 0.01 sin(i); 1e-4 abs + 1e-4 rel."""
    g = golden[dtype]
    columns = g["elements"] * blocks
    rows = 5 // blocks
    weight = clq.make_tensor_view(clq.make_packed_storage(dtype, g["bytes"]), (rows, columns))
    w64 = g["values"].astype(np.float64).reshape(rows, columns)
    for batch in (1, 3, 9):
        x = (0.01 * np.sin(np.arange(batch * columns))).astype(np.float32).reshape(batch, columns)
        got = clq.linear(x, weight)
        ref = x.astype(np.float64) @ w64.T
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - ref) <= 1e-4 + 1e-4 * np.abs(ref))


@pytest.mark.parametrize("dtype", DTYPES)
def test_nonfinite_scales_are_rejected(cuda, clq, golden, dtype):
    """tests/local/packed.lisp:48-52 and tests/mlx-gguf/kernels.lisp:104-111."""
    g = golden[dtype]
    k = g["elements"]
    for offset in g["bad_offsets"]:
        bad = g["bytes"].copy()
        bad[offset] = 0x7C
        weight = clq.make_tensor_view(clq.make_packed_storage(dtype, bad), (5, k))
        with pytest.raises(clq.ClqError) as err:
            clq.dequantize(weight)
        assert err.value.status == "CLQ_ERR_NONFINITE_SCALE"
        with pytest.raises(clq.ClqError) as err:
            clq.linear(np.ones((1, k), np.float32), weight)
        assert err.value.status == "CLQ_ERR_NONFINITE_SCALE"
        with pytest.raises(clq.ClqError):
            clq.Store(dtype, 5, k, bad)


def test_weights_upload_once_and_offset_views_reuse_them(cuda, clq, golden):
    lib = clq._lib.lib
    lib.clq_clear_cache()
    g = golden["q4_k"]
    storage = clq.make_q4_k_storage(g["bytes"].copy())
    weight = clq.make_tensor_view(storage, (5, 256))
    x = q8_activations(2, 256)
    first = clq.linear(x, weight)
    second = clq.linear(x, weight)
    assert np.array_equal(first, second)
    view = clq.make_tensor_view(storage, (3, 256), offset=2 * 256)
    third = clq.linear(x, view)
    assert np.array_equal(third, first[:, 2:])
    count, nbytes = ctypes.c_int64(), ctypes.c_int64()
    lib.clq_cache_stats(ctypes.byref(count), ctypes.byref(nbytes))
    assert count.value == 1 and nbytes.value == 5 * 144
    # copy-once: later writes to the host bytes are not seen (mlx-gguf/kernels.lisp:87-99)
    storage.bytes[143] ^= 0xFF
    assert np.array_equal(clq.linear(x, weight), first)
    del weight, view, storage
    import gc
    gc.collect()
    lib.clq_cache_stats(ctypes.byref(count), ctypes.byref(nbytes))
    assert count.value == 0


# ---- benchmark-configuration shapes ----------------------------------------

CONFIG_CASES = [
    # (config, dtype, n, k, m) -- shapes of the benchmark configurations
    (0, "q8_0", 4096, 4096, 1),
    (1, "q4_0", 2048, 2048, 1), (1, "q4_0", 512, 2048, 4), (1, "q4_0", 8192, 2048, 16),
    (1, "q4_0", 2048, 8192, 1),
    (1, "q4_k", 2048, 2048, 1), (1, "q4_k", 512, 2048, 4), (1, "q4_k", 8192, 2048, 16),
    (1, "q4_k", 2048, 8192, 4),
    (2, "q6_k", 4096, 4096, 1), (2, "q6_k", 1024, 4096, 8), (2, "q6_k", 12288, 4096, 64),
    (2, "q6_k", 4096, 12288, 8),
]


@pytest.mark.parametrize("config,dtype,n,k,m", CONFIG_CASES)
def test_config_shapes_against_oracle(cuda, clq, synth, oracle, config, dtype, n, k, m):
    data = synth.packed_blocks(dtype, n, k, seed=1000 * config + n % 997)
    x = synth.activations(m, k, seed=1000 * config + 500 + m)
    store = clq.Store(dtype, n, k, data)
    torch = cuda
    out = store.linear(torch.from_numpy(x).cuda()).cpu().numpy()
    # check a subset of rows against fp64 (the whole matrix when it is cheap)
    rows = n if n * k * m <= 64 * 2**20 else 1024
    sel = slice(0, rows)
    row_bytes = k // clq.DTYPES[dtype].block_size * clq.DTYPES[dtype].block_bytes
    ref, mag = oracle.matmul_f64(dtype, x, data[: rows * row_bytes], rows)
    assert max_row_relative_error(out[:, sel], ref) <= NORM_REL
    assert element_bound_ok(out[:, sel], ref, mag)
    store.close()


def test_vocab_projection_q6_k(cuda, clq, synth, oracle):
    """Q6_K output projection [128256 x 4096] at M = 1: full width, sampled rows checked."""
    torch = cuda
    n, k = 128256, 4096
    data = synth.packed_blocks("q6_k", n, k, seed=2001)
    x = synth.activations(1, k, seed=2002)
    store = clq.Store("q6_k", n, k, data)
    out = store.linear(torch.from_numpy(x).cuda()).cpu().numpy()
    rb = k // 256 * 210
    for start in (0, 64000, n - 512):
        ref, mag = oracle.matmul_f64("q6_k", x, data[start * rb:(start + 512) * rb], 512)
        assert element_bound_ok(out[:, start:start + 512], ref, mag)
    store.close()


@pytest.mark.parametrize("xtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("dtype", DTYPES)
def test_device_linear_shards_and_activation_types(cuda, clq, synth, oracle, dtype, xtype):
    """Row ranges (column-parallel shards) written into a wider output with a stride."""
    torch = cuda
    e = clq.DTYPES[dtype].block_size
    n, k, m = 300, 8 * e if e == 32 else 2 * e, 5
    data = synth.packed_blocks(dtype, n, k, seed=77)
    x = torch.from_numpy(synth.activations(m, k, seed=78)).cuda().to(getattr(torch, xtype))
    x32 = x.float().cpu().numpy()
    ref, mag = oracle.matmul_f64(dtype, x32, data, n)
    store = clq.Store(dtype, n, k, data)
    out = torch.full((m, n + 7), float("nan"), device="cuda")
    for begin, rows in ((0, 128), (128, 100), (228, 72)):
        store.linear(x, out=out[:, begin:begin + rows], row_begin=begin, rows=rows)
    got = out[:, :n].cpu().numpy()
    assert torch.isnan(out[:, n:]).all()
    assert element_bound_ok(got, ref, mag)
    store.close()


@pytest.mark.parametrize("dtype", DTYPES)
def test_activation_magnitudes_across_fp32_range(cuda, clq, synth, oracle, dtype):
    """Tiny, huge, zero and mixed activation rows keep the fp32-class bound."""
    torch = cuda
    n, k = 48, 1024
    data = synth.packed_blocks(dtype, n, k, seed=5)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((4, k)).astype(np.float32)
    x[0] *= np.float32(1e-30)
    x[1] *= np.float32(1e30)
    x[2, :512] = 0.0
    x[2, 512:] *= np.float32(1e4)
    x[3, ::7] *= np.float32(1e-6)
    ref, mag = oracle.matmul_f64(dtype, x, data, n)
    store = clq.Store(dtype, n, k, data)
    got = store.linear(torch.from_numpy(x).cuda()).cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - ref) <= 1e-5 * mag + 1e-37)
    store.close()


@pytest.mark.parametrize("dtype", DTYPES)
def test_grouped_launch_equals_separate_launches(cuda, clq, synth, oracle, dtype):
    """clq_linear_group_device: q/k/v-style members sharing x agree with one
    launch per member and match the oracle.  (A group partitions its tiles over
    the SMs differently from single launches; where that moves a K split
    between warps the sums round differently, so agreement is to fp32
    rounding, not bits.)"""
    torch = cuda
    k = 1024
    shapes = [512, 136, 136]
    datas = [synth.packed_blocks(dtype, n, k, seed=300 + i) for i, n in enumerate(shapes)]
    stores = [clq.Store(dtype, n, k, d) for n, d in zip(shapes, datas)]
    for m in (1, 3, 6):
        x = torch.from_numpy(synth.activations(m, k, seed=310 + m)).cuda()
        grouped = clq.linear_group(stores, x)
        for s, g, d, n in zip(stores, grouped, datas, shapes):
            single = s.linear(x)
            torch.testing.assert_close(single, g, rtol=1e-5, atol=1e-6)
            ref, mag = oracle.matmul_f64(dtype, x.cpu().numpy(), d, n)
            assert element_bound_ok(g.cpu().numpy(), ref, mag)
    for s in stores:
        s.close()
