"""The CPU oracle of the KV cache codec, RoPE and attention, pinned to the
reference's own cases (no GPU needed).

The Q8 cases are those of tests/local/cache.lisp (as the fixture
tests/golden/kv_golden.json, made from that file's text by
tests/golden/make_kv_golden.py): rounding and groups
(q8-cache-groups-rounding-and-overwrite), finite extrema
(q8-cache-reconstructs-finite-extrema), strided rows
(q8-cache-encodes-strided-rows) and non-finite rows
(q8-cache-rejects-nonfinite-values-and-invalid-options).  RoPE and attention
are checked against their definitions in local/blocks.lisp.
"""
import importlib
import json
import math
import pathlib

import numpy as np
import pytest

import attention as ref  # oracle/attention.py

# the reference's cases, read from tests/local/cache.lisp by tests/golden/make_kv_golden.py
KV = json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "kv_golden.json").read_text())
F32_MAX = np.finfo(np.float32).max
NONFINITE = {"single-float-positive-infinity": np.inf, "single-float-nan": np.nan}


def test_q8_rounding_groups_and_zero_scales():
    case = KV["rounding"]
    rows = np.array(case["row"], dtype=np.float32).reshape(case["shape"])
    codes, scales = ref.q8_store(rows)
    decoded = ref.q8_prefix(codes, scales).reshape(-1)
    assert decoded.tolist() == case["decoded"]
    assert scales.reshape(-1)[case["zero_group_index"]] == case["zero_group_scale"]  # all-zero group
    # the cache's buffers for n_ctx positions
    assert codes.size * case["n_ctx"] == case["bytes"] and scales.size * case["n_ctx"] == case["scales"]


def test_q8_reconstructs_finite_extrema():
    row = [F32_MAX if v == "most-positive-single-float" else -F32_MAX for v in KV["extrema"]["row"]]
    codes, scales = ref.q8_store(np.array(row, dtype=np.float32).reshape(1, 1, len(row)))
    decoded = ref.q8_prefix(codes, scales).reshape(-1)
    assert decoded.tolist() == [float(np.float32(v)) for v in row]


def test_q8_strided_rows_encode_as_their_copy():
    case = KV["strided"]
    source = np.arange(case["arange"], dtype=np.float32).reshape(case["shape"])
    rows = source.transpose(case["axes"])
    a = ref.q8_store(rows)
    b = ref.q8_store(np.ascontiguousarray(rows))
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


@pytest.mark.parametrize("name", KV["nonfinite"])
def test_q8_rejects_non_finite(name):
    with pytest.raises(ref.NonFinite):
        ref.q8_store(np.array([NONFINITE[name]], dtype=np.float32).reshape(1, 1, 1))


def test_rope_tables_and_pairings():
    cos, sin = ref.rope_tables(0, 3, 4, 10000.0)
    assert np.all(cos[0] == 1) and np.all(sin[0] == 0)  # position 0 is the identity
    assert cos[1, 0] == np.float32(math.cos(1.0)) and sin[2, 1] == np.float32(math.sin(2 * 0.01))
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 2, 6)).astype(np.float32)
    adj = ref.apply_rope(x, cos, sin, "adjacent", 4)
    neo = ref.apply_rope(x, cos, sin, "neox", 4)
    assert np.array_equal(adj[:, :, 4:], x[:, :, 4:]) and np.array_equal(neo[:, :, 4:], x[:, :, 4:])
    # adjacent pair i = (2i, 2i+1); neox pair i = (i, i + 2)
    p, h = 2, 1
    c, s = cos[p, 1], sin[p, 1]
    assert adj[p, h, 2] == x[p, h, 2] * c - x[p, h, 3] * s
    assert neo[p, h, 3] == x[p, h, 1] * s + x[p, h, 3] * c
    # the rotation keeps each pair's length
    n0 = np.hypot(x[:, :, 0:4:2], x[:, :, 1:4:2])
    n1 = np.hypot(adj[:, :, 0:4:2], adj[:, :, 1:4:2])
    assert np.allclose(n0, n1, rtol=1e-6)


def test_causal_mask_and_attention_definition():
    assert ref.causal_mask(2, 2, 0, 0).tolist() == [[True, False], [True, True]]
    assert ref.causal_mask(1, 3, 2, 0) is None  # a decode row sees every cached key
    rng = np.random.default_rng(1)
    keys = rng.standard_normal((5, 2, 8))
    values = rng.standard_normal((5, 2, 8))
    q = np.zeros((2, 4, 8))
    mask = ref.causal_mask(2, 5, 3, 0)
    out = ref.attend_f64(q, keys, values, mask, 4, 2)
    # zero queries: uniform weights over the visible keys; heads 0,1 read KV head 0
    assert np.allclose(out[0, 0:8], values[:4, 0].mean(axis=0))
    assert np.allclose(out[1, 8:16], values[:5, 0].mean(axis=0))
    assert np.allclose(out[1, 24:32], values[:5, 1].mean(axis=0))


def test_llama3_rope_factors_follow_the_reference_formula():
    att = importlib.import_module("cl-inference_b200.attention")
    scaling = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
               "original_max_position_embeddings": 8192}
    f = att.llama3_rope_factors(128, 500000.0, scaling)
    assert len(f) == 64 and f[0] == 1.0 and f[-1] == 8.0
    # a frequency in the smooth band
    i = next(j for j in range(64) if 8192 / 4 <= 2 * math.pi / 500000.0 ** (-2 * j / 128) <= 8192)
    w = 2 * math.pi / 500000.0 ** (-2 * i / 128)
    smooth = (8192 / w - 1) / 3
    assert f[i] == np.float32(1 / ((1 - smooth) / 8 + smooth))
    assert att.llama3_rope_factors(128, 500000.0, {"rope_type": "default"}) is None
    with pytest.raises(ValueError):
        att.llama3_rope_factors(128, 500000.0, {"rope_type": "yarn"})
    with pytest.raises(ValueError):
        att.llama3_rope_factors(128, 500000.0, dict(scaling, high_freq_factor=0.5))


@pytest.mark.parametrize("pairing", ["adjacent", "neox"])
def test_rope_is_relative(pairing):
    """Shifting every position leaves attention unchanged (tests/local/blocks.lisp,
    blocks-rope-is-relative): the rotation of q and k at positions p and p + 5
    gives the same scores up to the f32 rounding of the tables."""
    rng = np.random.default_rng(3)
    count, heads, kvh, hd = 2, 4, 2, 8
    q = rng.standard_normal((count, heads, hd)).astype(np.float32)
    k = rng.standard_normal((count, kvh, hd)).astype(np.float32)
    v = rng.standard_normal((count, kvh, hd)).astype(np.float32)
    outs = []
    for start in (0, 5):
        cos, sin = ref.rope_tables(start, count, hd, 10000.0)
        qr = ref.apply_rope(q, cos, sin, pairing, hd)
        kr = ref.apply_rope(k, cos, sin, pairing, hd)
        outs.append(ref.attend_f64(qr, kr, v, ref.causal_mask(count, count, start, start), heads, kvh))
    assert np.allclose(outs[0], outs[1], rtol=1e-5, atol=1e-5)
