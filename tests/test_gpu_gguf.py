"""GGUF file -> device store (clq_gguf_store), needs a B200.

Tensors of all four packed types go from a GGUF file through the chunked,
page-locked upload into stores; their device dequantization must equal the
gguf package's decoder (which matches the reference's goldens bit for bit)
and the oracle, and their products the oracle within the reference's bound.
A tensor larger than the staging chunk exercises both staging buffers; a
non-finite scale in the file fails at load (the scan of
mlx/gguf/weights.lisp:19-23); a non-packed tensor is refused.
"""
import importlib

import numpy as np
import pytest

import gguf_build as gb
from helpers import NORM_REL, element_bound_ok, max_row_relative_error

pytestmark = pytest.mark.gpu

SHAPES = {"q4_0": (96, 512), "q8_0": (64, 1024), "q4_k": (80, 1024), "q6_k": (48, 768)}


@pytest.fixture(scope="module")
def g():
    return importlib.import_module("cl-inference_b200.gguf")


def test_stores_from_file_match_decoder_and_oracle(cuda, clq, synth, oracle, g, tmp_path):
    torch = cuda
    gguf = pytest.importorskip("gguf")
    datas = {dt: synth.packed_blocks(dt, n, k, seed=50 + i) for i, (dt, (n, k)) in enumerate(SHAPES.items())}
    tensors = [(f"w.{dt}", (k, n), gb.GGML[dt], datas[dt]) for dt, (n, k) in SHAPES.items()]
    tensors.append(("norm", (16,), 0, gb.f32_bytes(range(16))))
    path = tmp_path / "m.gguf"
    path.write_bytes(gb.build(metadata=[("general.architecture", 8, "llama")], tensors=tensors))
    with g.GGUFFile(path) as f:
        for dt, (n, k) in SHAPES.items():
            store = f.store(f"w.{dt}")
            assert (store.n, store.k) == (n, k)
            dev = store.dequantize().cpu().numpy()
            want = gguf.quants.dequantize(datas[dt].reshape(n, -1), getattr(gguf.GGMLQuantizationType, dt.upper()))
            assert np.array_equal(dev.view(np.uint32), np.asarray(want, np.float32).reshape(n, k).view(np.uint32))
            x = synth.activations(3, k, seed=60)
            ref, mag = oracle.matmul_f64(dt, x, datas[dt], n)
            got = store.linear(torch.from_numpy(x).cuda()).cpu().numpy()
            assert max_row_relative_error(got, ref) <= NORM_REL
            assert element_bound_ok(got, ref, mag)
            store.close()
        with pytest.raises(clq.ClqError) as err:
            f.store("norm")
        assert err.value.status == "CLQ_ERR_UNSUPPORTED"


def test_multi_chunk_upload(cuda, clq, synth, g, tmp_path):
    """A 37.7 MB Q4_K tensor: three 16 MB chunks through the two staging buffers."""
    n, k = 16384, 4096
    data = synth.packed_blocks("q4_k", n, k, seed=71)
    path = tmp_path / "big.gguf"
    path.write_bytes(gb.build(tensors=[("big", (k, n), 12, data)]))
    with g.GGUFFile(path) as f:
        assert f.tensors["big"].nbytes == data.size and data.size > 2 * (16 << 20)
        store = f.store("big")
        ref = clq.Store("q4_k", n, k, data)
        for r0 in (0, 7000, n - 64):
            a = store.dequantize(row_begin=r0, rows=64).cpu().numpy()
            b = ref.dequantize(row_begin=r0, rows=64).cpu().numpy()
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        store.close()
        ref.close()


@pytest.mark.parametrize("dtype,scale_at", [("q8_0", 1), ("q4_k", 3), ("q6_k", 209)])
def test_non_finite_scale_fails_at_load(cuda, clq, synth, g, tmp_path, dtype, scale_at):
    n, k = 4, 256
    data = synth.packed_blocks(dtype, n, k, seed=3).copy()
    block = clq.DTYPES[dtype].block_bytes
    data[2 * block + scale_at] = 0x7C  # exponent 31 in the high byte of an fp16 scale
    path = tmp_path / "nan.gguf"
    path.write_bytes(gb.build(tensors=[("w", (k, n), gb.GGML[dtype], data)]))
    with g.GGUFFile(path) as f, pytest.raises(clq.ClqError) as err:
        f.store("w")
    assert err.value.status == "CLQ_ERR_NONFINITE_SCALE"


def test_load_rate(cuda, clq, g, tmp_path, capsys):
    """Upload rate from a page-cached file: eight 66 MB Q4_K tensors (the
    gate/up shape of Llama-3-8B), reported, not gated."""
    import time
    torch = cuda
    n, k = 14336 * 2, 4096
    nbytes = n * k // 256 * 144
    tensors = []
    gen = torch.Generator(device="cuda")
    for i in range(8):
        gen.manual_seed(90 + i)
        raw = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda", generator=gen)
        raw = raw.view(-1, 144)
        raw[:, 1] &= 0x3B  # finite, modest fp16 d and dmin (exponent < 31)
        raw[:, 3] &= 0x3B
        tensors.append((f"w{i}", (k, n), 12, raw.reshape(-1).cpu().numpy()))
    path = tmp_path / "rate.gguf"
    path.write_bytes(gb.build(tensors=tensors))
    with g.GGUFFile(path) as f:
        f.store("w0").close()  # staging set up, file pages touched once
        t0 = time.perf_counter()
        stores = [f.store(name) for name in f.tensors]
        torch.cuda.synchronize()
        sec = time.perf_counter() - t0
        for s in stores:
            s.close()
    with capsys.disabled():
        print(f"\nGGUF -> device stores: {8 * nbytes / sec / 1e9:.2f} GB/s ({8 * nbytes / 1e6:.0f} MB in {sec * 1e3:.1f} ms)")
