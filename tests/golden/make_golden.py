"""Regenerate tests/golden/quant_golden.json from the cl-inference sources.

Reads, as text, the llama.cpp golden blocks in the reference's
tests/local/quant-golden.lisp:3-17 (Q4_0, Q4_K, Q6_K: five blocks each, with the
values llama.cpp 8bb3cf0 `dequantize_row_*` produced) and rebuilds the Q8_0
golden of tests/mlx-gguf/kernels.lisp:9-21 from its stated formula.  Every
value is stored as its little-endian IEEE-754 bytes (hex) so that signed
zeros survive.

The third-party decoder `gguf.quants.dequantize` (llama.cpp's Python package,
when importable) is run over the same bytes as an independent cross-check and
its agreement is recorded in the fixture.

Usage: python tests/golden/make_golden.py /path/to/cl-inference
Only this script reads the reference checkout; tests read the JSON it writes.
"""
import json
import pathlib
import re
import struct
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def lisp_float(token):
    # "2.5f0", "-4.76837158f-07" -> python float (single-float literals)
    return float(token.replace("f", "e"))


def parse_packed_goldens(text):
    """Return {dtype: (bytes, float32 values)} from quant-golden.lisp."""
    out = {}
    pattern = re.compile(r"\(:(q4_0|q4_k|q6_k)\s+#\(([^)]*)\)\s+#\(([^)]*)\)\)", re.S)
    for match in pattern.finditer(text):
        dtype = match.group(1)
        raw = bytes(int(v) for v in match.group(2).split())
        values = np.array([lisp_float(v) for v in match.group(3).split()], dtype=np.float32)
        out[dtype] = (raw, values)
    if set(out) != {"q4_0", "q4_k", "q6_k"}:
        raise RuntimeError(f"expected three packed goldens, found {sorted(out)}")
    return out


def q8_golden():
    """tests/mlx-gguf/kernels.lisp:9-21: five Q8_0 blocks, code ((i*73+block*19) mod 256) - 128."""
    scales = [0.0, 0.5, -2.0, 0.00006103515625, 8.0]
    bits = [0, 0x3800, 0xC000, 0x0400, 0x4800]
    raw = bytearray(170)
    expected = np.zeros(160, dtype=np.float32)
    for block, (scale, encoding) in enumerate(zip(scales, bits)):
        raw[block * 34] = encoding & 255
        raw[block * 34 + 1] = encoding >> 8
        for i in range(32):
            code = ((i * 73 + block * 19) % 256) - 128
            raw[block * 34 + 2 + i] = code & 255
            expected[block * 32 + i] = np.float32(scale) * np.float32(code)
    return bytes(raw), expected


def gguf_cross_check(dtype, raw, values):
    try:
        import gguf.quants as gq
        from gguf import GGMLQuantizationType as T
    except Exception as exc:  # pragma: no cover - depends on the environment
        return f"gguf unavailable: {exc}"
    qtype = {"q4_0": T.Q4_0, "q8_0": T.Q8_0, "q4_k": T.Q4_K, "q6_k": T.Q6_K}[dtype]
    decoded = gq.dequantize(np.frombuffer(raw, dtype=np.uint8), qtype).astype(np.float32).ravel()
    same = np.array_equal(decoded.view(np.uint32), np.asarray(values, np.float32).view(np.uint32))
    return "bit-identical" if same else "DIFFERS"


def main():
    if len(sys.argv) != 2:
        raise SystemExit(f"usage: python {sys.argv[0]} /path/to/cl-inference")
    root = pathlib.Path(sys.argv[1])
    packed = parse_packed_goldens((root / "tests/local/quant-golden.lisp").read_text())
    raw8, values8 = q8_golden()
    fixtures = {"q8_0": (raw8, values8), **packed}
    geometry = {"q4_0": (32, 18, 2), "q8_0": (32, 34, 8), "q4_k": (256, 144, 12), "q6_k": (256, 210, 14)}
    # byte set to 0x7C (exponent 31) by the error-path tests:
    # tests/local/packed.lisp:48-52 and tests/mlx-gguf/kernels.lisp:104-111
    bad_offsets = {"q4_0": [1], "q8_0": [1], "q4_k": [1, 3], "q6_k": [209]}
    doc = {
        "provenance": {
            "q4_0/q4_k/q6_k": "tests/local/quant-golden.lisp:3-17 (llama.cpp 8bb3cf0 dequantize_row_*)",
            "q8_0": "tests/mlx-gguf/kernels.lisp:9-21 (scale * code)",
            "generator": "tests/golden/make_golden.py",
        },
        "fixtures": {},
    }
    for dtype, (raw, values) in fixtures.items():
        elements, block_bytes, ggml_id = geometry[dtype]
        assert len(raw) == 5 * block_bytes and len(values) == 5 * elements, dtype
        doc["fixtures"][dtype] = {
            "ggml_type": ggml_id,
            "elements": elements,
            "block_bytes": block_bytes,
            "blocks": 5,
            "bytes_hex": bytes(raw).hex(),
            "value_bits_hex": np.asarray(values, "<f4").tobytes().hex(),
            "nonfinite_scale_offsets": bad_offsets[dtype],
            "gguf_quants_cross_check": gguf_cross_check(dtype, raw, values),
        }
    (HERE / "quant_golden.json").write_text(json.dumps(doc, indent=1) + "\n")
    for dtype, entry in doc["fixtures"].items():
        print(dtype, entry["gguf_quants_cross_check"])


if __name__ == "__main__":
    main()
