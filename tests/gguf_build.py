"""A test-only GGUF v3 writer whose knobs make the malformed files a reader must
reject (the cases of the reference's tests/local/gguf.lisp)."""
import struct

GGML = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 8, "q4_k": 12, "q6_k": 14, "bf16": 30}


def _uint(value, size):
    return (value & ((1 << (8 * size)) - 1)).to_bytes(size, "little")


def _string(s):
    raw = s.encode() if isinstance(s, str) else bytes(s)
    return _uint(len(raw), 8) + raw


def _value(vtype, value):
    """VTYPE is a GGUF value type id; arrays are ("array", element type, items)."""
    if vtype in (0, 1):
        return _uint(value, 1)
    if vtype in (2, 3):
        return _uint(value, 2)
    if vtype in (4, 5, 99):
        return _uint(value, 4)
    if vtype == 6:
        return struct.pack("<f", value)
    if vtype == 7:
        return _uint(value if isinstance(value, int) and not isinstance(value, bool) else int(bool(value)), 1)
    if vtype == 8:
        return _string(value)
    if vtype == 9:
        _, etype, items = value
        return _uint(etype, 4) + _uint(len(items), 8) + b"".join(_value(etype, it) for it in items)
    if vtype in (10, 11):
        return _uint(value, 8)
    if vtype == 12:
        return struct.pack("<d", value)
    raise ValueError(vtype)


def nested_array(depth):
    """An array of arrays DEPTH levels deep, ending in an empty array."""
    return ("array", 0, []) if depth == 0 else ("array", 9, [nested_array(depth - 1)])


def build(metadata=(), tensors=(), alignment=32, version=3, magic=0x46554747, tensor_count=None,
          truncate=0, pad=True):
    """METADATA: (key, type, value) triples.  TENSORS: (name, dims in file order,
    ggml type id, bytes[, offset]); offsets default to the next aligned slot."""
    metadata = list(metadata)
    if alignment != 32:
        metadata.append(("general.alignment", 4, alignment))
    head = bytearray()
    head += _uint(magic, 4) + _uint(version, 4)
    head += _uint(len(tensors) if tensor_count is None else tensor_count, 8) + _uint(len(metadata), 8)
    for key, vtype, value in metadata:
        head += _string(key) + _uint(vtype, 4) + _value(vtype, value)
    data = bytearray()
    cursor = 0
    for t in tensors:
        name, dims, type_id, raw = t[:4]
        offset = t[4] if len(t) > 4 else cursor
        head += _string(name) + _uint(len(dims), 4) + b"".join(_uint(d, 8) for d in dims)
        head += _uint(type_id, 4) + _uint(offset, 8)
        if len(data) < offset:
            data += bytes(offset - len(data))
        raw = bytes(raw)
        end = offset + len(raw)
        if len(data) < end:
            data += bytes(end - len(data))
        data[offset:end] = raw
        cursor = -(-len(data) // alignment) * alignment
    if pad:
        head += bytes(-len(head) % alignment)
    out = bytes(head + data)
    return out[:len(out) - truncate] if truncate else out


def f32_bytes(values):
    return b"".join(struct.pack("<f", v) for v in values)


def u16_bytes(values):
    return b"".join(_uint(v, 2) for v in values)
