"""GGUF reader of libclq (clq_gguf_*), no GPU needed.

Mirrors tests/local/gguf.lisp: the sample file's listing, shapes and bytes,
every metadata value type, custom alignment, and every malformed file the
reference rejects (CLQ_ERR_FORMAT).  A file written by the gguf package
(0.19.0) is also read back against gguf.GGUFReader.
"""
import importlib

import numpy as np
import pytest

import gguf_build as gb

Q8_BLOCK = gb.u16_bytes([0x3C00]) + bytes((i - 16) & 0xFF for i in range(32))
Q4K_BLOCK = bytes([7]) * 144


@pytest.fixture(scope="module")
def mod():
    return importlib.import_module("cl-inference_b200.gguf"), importlib.import_module("cl-inference_b200._lib")


def sample(**overrides):
    return gb.build(metadata=[("general.architecture", 8, "llama")],
                    tensors=[("f32", (3, 2), 0, gb.f32_bytes([0, 1, 2, 3, 4, 5])),
                             ("f16", (2,), 1, gb.u16_bytes([0x3C00, 0x4000])),
                             ("bf16", (2,), 30, gb.u16_bytes([0x3F80, 0x4000])),
                             ("q8", (32,), 8, Q8_BLOCK),
                             ("q4k", (256,), 12, Q4K_BLOCK)], **overrides)


def write(tmp_path, data, name="t.gguf"):
    p = tmp_path / name
    p.write_bytes(data)
    return p


def open_bad(mod, tmp_path, data):
    g, lib = mod
    with pytest.raises(lib.ClqError) as err:
        g.GGUFFile(write(tmp_path, data, "bad.gguf"))
    assert err.value.status == "CLQ_ERR_FORMAT", str(err.value)


def test_listing_shapes_and_bytes(mod, tmp_path):
    g, _ = mod
    with g.GGUFFile(write(tmp_path, sample())) as f:
        assert list(f.tensors) == ["f32", "f16", "bf16", "q8", "q4k"]
        info = f.tensors["f32"]
        assert info.shape == (2, 3) and info.ggml_type == 0 and info.nbytes == 24
        assert f.tensors["q8"].nbytes == 34 and f.tensors["q4k"].nbytes == 144
        vals = np.frombuffer(f.tensor_bytes("f32").tobytes(), np.float32).reshape(2, 3)
        assert vals[1, 0] == 3 and vals[1, 2] == 5  # row-major, as the f32 view
        assert f.tensor_bytes("q8").tobytes() == Q8_BLOCK
        assert f.tensor_bytes("q4k").tobytes() == Q4K_BLOCK
        assert f.metadata("general.architecture") == "llama"
        assert not f.tensor_bytes("q8").flags.writeable


def test_metadata_value_types(mod, tmp_path):
    g, _ = mod
    data = gb.build(metadata=[("u8", 0, 200), ("i8", 1, -3), ("u16", 2, 60000), ("i16", 3, -300),
                              ("u32", 4, 4000000000), ("i32", 5, -5), ("f32", 6, 1.5), ("bool", 7, True),
                              ("str", 8, "héllo"), ("u64", 10, 18446744073709551615), ("i64", 11, -7),
                              ("f64", 12, 2.25), ("u32s", 9, ("array", 4, [1, 2, 3])),
                              ("f32s", 9, ("array", 6, [0.5, -1.5])), ("strs", 9, ("array", 8, ["a", "bc"])),
                              ("nested", 9, ("array", 9, [("array", 4, [1]), ("array", 4, [2, 3])]))])
    with g.GGUFFile(write(tmp_path, data)) as f:
        m = f.metadata
        assert (m("u8"), m("i8"), m("u16"), m("i16")) == (200, -3, 60000, -300)
        assert (m("u32"), m("i32"), m("f32"), m("bool")) == (4000000000, -5, 1.5, True)
        assert m("str") == "héllo" and m("u64") == 18446744073709551615 and m("i64") == -7 and m("f64") == 2.25
        assert m("u32s") == ("array", "u32", 3) and m("f32s") == ("array", "f32", 2)
        assert m("strs") == ("array", "str", 2) and m("nested") == ("array", "array", 2)
        assert f.keys[:2] == ["u8", "i8"]
        assert not f.tensors


def test_custom_alignment(mod, tmp_path):
    g, _ = mod
    with g.GGUFFile(write(tmp_path, sample(alignment=64))) as f:
        vals = np.frombuffer(f.tensor_bytes("f32").tobytes(), np.float32)
        assert vals[5] == 5
        assert f.tensor_bytes("q8").tobytes() == Q8_BLOCK


def test_files_without_tensors_need_no_padding(mod, tmp_path):
    g, _ = mod
    with g.GGUFFile(write(tmp_path, gb.build(metadata=[("general.architecture", 8, "llama")], pad=False))) as f:
        assert f.metadata("general.architecture") == "llama" and not f.tensors


def test_rejects_empty_short_and_bad_headers(mod, tmp_path):
    for data in (b"", sample()[:10], sample(magic=0x12345678), sample(version=2), sample(version=0x03000000)):
        open_bad(mod, tmp_path, data)


def test_rejects_truncation(mod, tmp_path):
    for data in (sample(truncate=1), sample()[:60], sample(tensor_count=1000000),
                 gb.build(tensors=[("t", (1,), 0, gb.f32_bytes([1.0]))], truncate=5)):
        open_bad(mod, tmp_path, data)


def test_rejects_duplicates(mod, tmp_path):
    open_bad(mod, tmp_path, gb.build(metadata=[("k", 4, 1), ("k", 4, 2)]))
    two = gb.f32_bytes([1.0, 2.0])
    open_bad(mod, tmp_path, gb.build(tensors=[("t", (2,), 0, two), ("t", (2,), 0, two)]))


def test_nesting_limit(mod, tmp_path):
    g, _ = mod
    with g.GGUFFile(write(tmp_path, gb.build(metadata=[("n", 9, gb.nested_array(30))]))) as f:
        assert f.metadata("n")[0] == "array"
    open_bad(mod, tmp_path, gb.build(metadata=[("n", 9, gb.nested_array(40))]))


def test_rejects_invalid_values(mod, tmp_path):
    open_bad(mod, tmp_path, gb.build(metadata=[("b", 7, 2)]))
    open_bad(mod, tmp_path, gb.build(metadata=[("u", 99, 1)]))
    open_bad(mod, tmp_path, gb.build(metadata=[("s", 8, bytes([255, 254]))]))


def test_rejects_invalid_alignment(mod, tmp_path):
    open_bad(mod, tmp_path, sample(alignment=48))
    open_bad(mod, tmp_path, sample(alignment=8192))
    open_bad(mod, tmp_path, gb.build(metadata=[("general.alignment", 6, 32.0)]))


def test_rejects_bad_tensors(mod, tmp_path):
    four = gb.f32_bytes([1.0, 2.0, 3.0, 4.0])
    for dims, typ, extra in (((), 0, ()), ((1, 1, 1, 1, 1), 0, ()), ((0,), 0, ()), ((4,), 99, ()),
                             ((4,), 4, ()), ((33,), 8, ()), ((4,), 0, (1,))):
        open_bad(mod, tmp_path, gb.build(tensors=[("t", dims, typ, four) + tuple(extra)]))


def test_rejects_overlapping_tensors(mod, tmp_path):
    four = gb.f32_bytes([1.0, 2.0, 3.0, 4.0])
    open_bad(mod, tmp_path, gb.build(tensors=[("a", (4,), 0, four, 0), ("b", (4,), 0, four, 0)]))


def test_rejects_offsets_that_wrap_past_the_end(mod, tmp_path):
    """A tensor whose aligned offset sits just below 2^64 would pass a check of
    data_start + offset + nbytes against the file size once the sum wraps; the
    reader rejects it like any tensor past the end of the file."""
    four = gb.f32_bytes([1.0, 2.0, 3.0, 4.0])
    good = gb.build(tensors=[("t", (4,), 0, four, 0)])
    # the tensor record ends with its u64 offset (0) right before the header padding
    rec = gb._string("t") + gb._uint(1, 4) + gb._uint(4, 8) + gb._uint(0, 4)
    at = good.index(rec) + len(rec)
    assert good[at:at + 8] == bytes(8)
    for offset in (2**64 - 32, 2**64 - 4096, 2**63):
        bad = good[:at] + gb._uint(offset, 8) + good[at + 8:]
        open_bad(mod, tmp_path, bad)


def test_missing_file_is_an_io_error(mod, tmp_path):
    g, lib = mod
    with pytest.raises(lib.ClqError) as err:
        g.GGUFFile(tmp_path / "absent.gguf")
    assert err.value.status == "CLQ_ERR_IO"


def test_matches_the_gguf_package_reader(mod, tmp_path, synth):
    """A file written by gguf.GGUFWriter reads back as gguf.GGUFReader reads it."""
    gguf = pytest.importorskip("gguf")
    g, _ = mod
    rng = np.random.default_rng(5)
    path = tmp_path / "w.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_uint32("llama.block_count", 2)
    w.add_string("tokenizer.ggml.model", "gpt2")
    f32 = rng.standard_normal((3, 64)).astype(np.float32)
    w.add_tensor("norm", f32)
    q8 = gguf.quants.quantize(rng.standard_normal((4, 64)).astype(np.float32), gguf.GGMLQuantizationType.Q8_0)
    w.add_tensor("q8", q8, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    q4k = synth.packed_blocks("q4_k", 6, 512, seed=7).reshape(6, -1)
    w.add_tensor("q4k", q4k, raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    q6k = synth.packed_blocks("q6_k", 3, 256, seed=8).reshape(3, -1)
    w.add_tensor("q6k", q6k, raw_dtype=gguf.GGMLQuantizationType.Q6_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    ref = gguf.GGUFReader(str(path))
    with g.GGUFFile(path) as f:
        assert list(f.tensors) == [t.name for t in ref.tensors]
        for t in ref.tensors:
            info = f.tensors[t.name]
            assert info.ggml_type == int(t.tensor_type)
            assert info.shape == tuple(int(d) for d in reversed(t.shape))
            assert info.nbytes == int(t.n_bytes)
            assert f.tensor_bytes(t.name).tobytes() == np.asarray(t.data).tobytes()
        assert f.metadata("llama.block_count") == 2
        assert f.metadata("tokenizer.ggml.model") == "gpt2"
        assert f.metadata("general.architecture") == "llama"


@pytest.mark.parametrize("dtype", ["q4_0", "q4_k", "q6_k", "q8_0"])
def test_golden_blocks_through_a_gguf_file(mod, tmp_path, golden, oracle, dtype):
    """tests/local/packed.lisp, packed-gguf-uses-mapped-storage: the golden
    blocks written as a GGUF tensor read back as the same bytes (from the
    mapping) and decode (the oracle here; the device in tests/test_gpu_gguf.py)
    to the golden values bit for bit."""
    g, _ = mod
    gd = golden[dtype]
    nblocks = gd["bytes"].size // gd["block_bytes"]
    path = write(tmp_path, gb.build(tensors=[("packed", (gd["elements"], nblocks), gd["ggml_type"], gd["bytes"])]))
    with g.GGUFFile(path) as f:
        info = f.tensors["packed"]
        assert info.ggml_type == gd["ggml_type"] and info.shape == (nblocks, gd["elements"])
        raw = f.tensor_bytes("packed")
        assert raw.tobytes() == gd["bytes"].tobytes()
        out = np.asarray(oracle.dequantize(dtype, raw), np.float32)
        assert np.array_equal(out.view(np.uint32), gd["values"].view(np.uint32))
