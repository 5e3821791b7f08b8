"""Packed storage and view rules of the host mirror (CPU only).

Mirrors the storage/view rejections of tests/local/packed.lisp:41-47,61 and
tests/local/quant.lisp:77-98; no GPU work happens here.
"""
import numpy as np
import pytest

DTYPES = ["q8_0", "q4_0", "q4_k", "q6_k"]


@pytest.mark.parametrize("dtype", DTYPES)
def test_storage_and_view_rules(clq, golden, dtype):
    g = golden[dtype]
    k = g["elements"]
    storage = clq.make_packed_storage(dtype, g["bytes"])
    assert storage.storage_length == 5 * k
    weight = clq.make_tensor_view(storage, (5, k))
    with pytest.raises(clq.PackedError):
        clq.make_tensor_view(storage, (5, k - 1))
    with pytest.raises(clq.PackedError):
        clq.make_tensor_view(storage, (4, k), offset=1)
    with pytest.raises(clq.PackedError):
        clq.make_packed_storage(dtype, g["bytes"][:-1])
    with pytest.raises(clq.PackedError):
        clq.make_packed_storage(dtype, np.array([1, 2, 3], np.uint8))
    with pytest.raises(clq.PackedError):
        clq.make_packed_storage(dtype, g["bytes"].astype(np.int16))
    # an offset view of whole rows is fine
    view = clq.make_tensor_view(storage, (3, k), offset=k)
    assert view.byte_offset() == g["block_bytes"]
    # weight must be on the right and transposed (tests/local/packed.lisp:61)
    x = np.zeros((5, k), np.float32)
    with pytest.raises(clq.UnsupportedOperation):
        clq.matmul(clq.transpose(weight), x)
    with pytest.raises(clq.UnsupportedOperation):
        clq.matmul(x[:, :k], weight)
    with pytest.raises(clq.UnsupportedOperation):
        clq.astype(weight, "f64")
    assert clq.transpose(weight).transposed_matrix_p()


def test_q8_views_are_whole_blocks(clq):
    storage = clq.make_q8_0_storage(np.zeros(8 * 34, np.uint8))
    assert storage.storage_length == 256
    with pytest.raises(clq.PackedError):
        clq.make_tensor_view(storage, (4, 16))
    with pytest.raises(clq.PackedError):
        clq.make_tensor_view(storage, (3, 64), offset=16)
    with pytest.raises(clq.PackedError):
        clq.make_tensor_view(storage, (64, 4))
    assert clq.make_tensor_view(storage, (2, 64), offset=128).shape == (2, 64)
    with pytest.raises(clq.PackedError):
        clq.make_q8_0_storage(np.zeros(35, np.uint8))
    # the Q8_0 matmul needs a zero-offset weight (quant/q8-0.lisp:62-67)
    w = clq.make_tensor_view(storage, (2, 64), offset=128)
    with pytest.raises(clq.UnsupportedOperation):
        clq.matmul(np.zeros((1, 64), np.float32), clq.transpose(w))


def test_take_keeps_the_packed_dtype(clq, golden):
    g = golden["q4_k"]
    weight = clq.make_tensor_view(clq.make_q4_k_storage(g["bytes"]), (5, 256))
    taken = clq.take(weight, [4, 1, 4])
    assert taken.dtype.name == "q4_k" and taken.shape == (3, 256)
    rb = 144
    assert np.array_equal(taken.storage.bytes[:rb], g["bytes"][4 * rb:5 * rb])
    assert np.array_equal(taken.storage.bytes[rb:2 * rb], g["bytes"][rb:2 * rb])
    with pytest.raises(clq.PackedError):
        clq.take(weight, [5])
    copied = clq.copy_tensor(weight)
    assert np.array_equal(copied.storage.bytes, g["bytes"])
