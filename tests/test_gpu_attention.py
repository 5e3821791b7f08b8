"""KV cache, RoPE and attention on the device against the oracle (needs a B200).

The Q8 codec must give the oracle's codes and scales bit for bit (checked
through the decoded prefix), over random rows, all-zero groups, odd head
widths, strided rows and the finite extrema; f32 caches return what was
stored.  RoPE matches the oracle's tables and rotation to the last bit or one
ulp (double-precision cos and sin rounded to f32).  Attention over the cached
prefix matches the float64 restatement of attend with the causal mask within
1e-5 of the output's scale, for decode rows, a chunk of prompt rows, grouped
heads of 4, 8 and 16 and the small heads of the reference's tests, in every
form of the kernel: blocks of 1 to 16 query rows per CTA (ragged last
blocks), one position range written directly or several merged by a second
launch, and f32 key and value rows staged by bulk copies or by vector loads
(CLQ_ATTN_BULK=0, Q8 caches and odd head widths).  Past-context
updates fail with CLQ_ERR_CONTEXT and non-finite Q8 rows with
CLQ_ERR_NONFINITE_VALUE (local/kv-cache.lisp:49,94-96).
"""
import importlib

import numpy as np
import pytest

import attention as ref  # oracle/attention.py

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def att():
    return importlib.import_module("cl-inference_b200.attention")


def ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


@pytest.mark.parametrize("dim", [128, 35, 8])
def test_q8_cache_matches_the_codec(cuda, att, dim):
    torch = cuda
    rng = np.random.default_rng(dim)
    heads, n = 3, 40
    rows = (rng.standard_normal((n, heads, dim)) * np.exp(rng.uniform(-20, 20, (n, heads, 1)))).astype(np.float32)
    rows[5, 1, :] = 0.0                      # an all-zero head row
    rows[7, 0, : min(32, dim)] = 0.0         # an all-zero group
    rows[9, 2, 0] = np.float32(np.finfo(np.float32).max)
    rows[9, 2, 1 % dim] = -np.float32(np.finfo(np.float32).max)
    with att.KVCache(64, 2, heads, dim, "q8") as cache:
        x = torch.from_numpy(rows).cuda()
        cache.update(1, x[:25], x[:25] * 0.5, 0, check=True)
        cache.update(1, x[25:], x[25:] * 0.5, 25, check=True)
        keys, values = cache.prefix(1, n)
        kc, ks = ref.q8_store(rows)
        vc, vs = ref.q8_store(rows * np.float32(0.5))
        assert np.array_equal(keys.cpu().numpy().view(np.uint32), ref.q8_prefix(kc, ks).view(np.uint32))
        assert np.array_equal(values.cpu().numpy().view(np.uint32), ref.q8_prefix(vc, vs).view(np.uint32))
        # layer 0 untouched: codes 0, scales 1
        k0, _ = cache.prefix(0, n)
        assert float(k0.abs().max()) == 0.0


def test_q8_rounding_case_and_strided_rows(cuda, att):
    torch = cuda
    values = [127.0, -127.0, 0.5, 1.5, 2.5, -0.5, -1.5] + [0.0] * 28
    with att.KVCache(3, 1, 1, 35, "q8") as cache:
        row = torch.tensor(values, dtype=torch.float32, device="cuda").view(1, 1, 35)
        cache.update(0, row, row, 0, check=True)
        keys, _ = cache.prefix(0, 1)
        assert keys.view(35).tolist() == [127.0, -127.0, 0.0, 2.0, 2.0, 0.0, -2.0] + [0.0] * 28
        # overwrite position 0 with zeros after filling position 1
        cache.update(0, row, row, 1, check=True)
        zero = torch.zeros(1, 1, 35, device="cuda")
        cache.update(0, zero, zero, 0, check=True)
        keys, _ = cache.prefix(0, 1)
        assert float(keys.abs().max()) == 0.0
    source = torch.arange(210, dtype=torch.float32, device="cuda").view(2, 3, 35)
    rows = source.transpose(0, 1)  # (3, 2, 35), position stride 35, head stride 105
    with att.KVCache(3, 1, 2, 35, "q8") as a, att.KVCache(3, 1, 2, 35, "q8") as b:
        a.update(0, rows, rows, 0, check=True)
        copy = rows.contiguous()
        b.update(0, copy, copy, 0, check=True)
        assert torch.equal(a.prefix(0, 3)[0], b.prefix(0, 3)[0])


def test_cache_errors(cuda, att, clq):
    torch = cuda
    with att.KVCache(4, 1, 1, 1, "q8") as cache:
        for bad in (float("inf"), float("nan")):
            row = torch.tensor([bad], dtype=torch.float32, device="cuda").view(1, 1, 1)
            with pytest.raises(clq.ClqError) as err:
                cache.update(0, row, row, 0, check=True)
            assert err.value.status == "CLQ_ERR_NONFINITE_VALUE"
        assert cache.status() == 0
        ok = torch.ones(2, 1, 1, device="cuda")
        with pytest.raises(clq.ClqError) as err:
            cache.update(0, ok, ok, 3)
        assert err.value.status == "CLQ_ERR_CONTEXT"
    with pytest.raises(clq.ClqError):
        att.KVCache(4, 1, 1, 1, "q4")


def test_f32_cache_round_trip(cuda, att):
    torch = cuda
    x = torch.randn(10, 4, 64, device="cuda")
    with att.KVCache(16, 3, 4, 64, "f32") as cache:
        cache.update(2, x, -x, 3)
        k, v = cache.prefix(2, 13)
        assert torch.equal(k[3:13], x) and torch.equal(v[3:13], -x) and float(k[:3].abs().max()) == 0.0


@pytest.mark.parametrize("pairing", ["adjacent", "neox"])
@pytest.mark.parametrize("rope_dims,factors", [(128, False), (64, False), (128, True)])
def test_rope_matches_tables(cuda, att, pairing, rope_dims, factors):
    torch = cuda
    rng = np.random.default_rng(rope_dims)
    count, heads, hd, start, theta = 5, 8, 128, 1000, 500000.0
    x = rng.standard_normal((count, heads, hd)).astype(np.float32)
    f = None
    if factors:
        scaling = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                   "original_max_position_embeddings": 8192}
        f = np.array(att.llama3_rope_factors(rope_dims, theta, scaling), dtype=np.float32)
    cos, sin = ref.rope_tables(start, count, rope_dims, theta, f)
    want = ref.apply_rope(x, cos, sin, pairing, rope_dims)
    dev = torch.from_numpy(x).cuda()
    att.rope(dev, start, theta, rope_dims, pairing, None if f is None else torch.from_numpy(f).cuda())
    got = dev.cpu().numpy()
    assert int(ulps(got, want).max()) <= 1
    assert np.mean(got.view(np.uint32) == want.view(np.uint32)) > 0.99


@pytest.mark.parametrize("cache_type", ["f32", "q8"])
@pytest.mark.parametrize("count,heads,kv,hd,end,qstart", [
    (1, 32, 8, 128, 1000, 999),    # decode at position 999, Llama-3-8B heads
    (1, 64, 8, 128, 300, 299),     # Llama-3-70B grouping (8 query heads per KV head)
    (6, 32, 8, 128, 70, 64),       # a chunk of prompt rows at positions 64..69 (causal)
    (4, 2, 1, 8, 4, 0),            # the reference tests' small heads
    (1, 16, 1, 64, 1024, 1023),    # 16 query heads per KV head
    (64, 32, 8, 128, 1024, 960),   # 64 prompt rows, 4 to a CTA
    (3, 32, 8, 128, 4000, 3997),   # a long prefix, three rows (a ragged block of 4)
    (5, 8, 8, 64, 40, 35),         # one query head per KV head: 8 rows to a CTA
    (2, 8, 2, 128, 12, 10),        # a prefix of one range: written without the merge
    (2, 4, 2, 36, 150, 148),       # a head width off the 16-column grid (scalar tail)
    (3, 8, 4, 96, 300, 297),       # a head width with no specialised kernel
])
def test_attention_matches_oracle(cuda, att, cache_type, count, heads, kv, hd, end, qstart):
    torch = cuda
    rng = np.random.default_rng(end + count)
    keys = rng.standard_normal((end, kv, hd)).astype(np.float32)
    vals = rng.standard_normal((end, kv, hd)).astype(np.float32)
    q = (rng.standard_normal((count, heads, hd)) * 2).astype(np.float32)
    with att.KVCache(max(1024, end), 2, kv, hd, cache_type) as cache:
        cache.update(1, torch.from_numpy(keys).cuda(), torch.from_numpy(vals).cuda(), 0, check=True)
        out = att.attend(torch.from_numpy(q).cuda(), cache, 1, end, qstart).cpu().numpy()
        k_used, v_used = (keys, vals)
        if cache_type == "q8":
            k_used = ref.q8_prefix(*ref.q8_store(keys))
            v_used = ref.q8_prefix(*ref.q8_store(vals))
        mask = ref.causal_mask(count, end, qstart, 0)
        want = ref.attend_f64(q, k_used, v_used, mask, heads, kv)
    scale = np.abs(want).max()
    assert np.abs(out - want).max() <= 1e-5 * scale
    assert np.linalg.norm(out - want) / np.linalg.norm(want) <= 1e-6 * 4


def test_attention_argument_checks(cuda, att, clq):
    torch = cuda
    with att.KVCache(8, 1, 2, 16, "f32") as cache:
        q = torch.zeros(1, 6, 16, device="cuda")
        with pytest.raises(clq.ClqError):
            att.attend(torch.zeros(1, 3, 16, device="cuda"), cache, 0, 4, 3)  # 3 heads over 2 KV heads
        with pytest.raises(clq.ClqError):
            att.attend(q, cache, 0, 9, 3)  # past the context
        with pytest.raises(clq.ClqError):
            att.attend(q, cache, 1, 4, 3)  # no such layer


@pytest.mark.parametrize("cache_type", ["f32", "q8"])
def test_cache_filled_in_chunks_matches_a_full_pass(cuda, att, cache_type):
    """tests/local/blocks.lisp, blocks-cache-matches-a-full-pass: rows stored 3,
    then 1, then 1 at a time and attended as they arrive give, for the last
    row, what one pass over all five rows gives."""
    torch = cuda
    rng = np.random.default_rng(9)
    heads, kv, hd, n = 4, 2, 32, 5
    keys = rng.standard_normal((n, kv, hd)).astype(np.float32)
    vals = rng.standard_normal((n, kv, hd)).astype(np.float32)
    q = rng.standard_normal((n, heads, hd)).astype(np.float32)
    k_used, v_used = keys, vals
    if cache_type == "q8":
        k_used = ref.q8_prefix(*ref.q8_store(keys))
        v_used = ref.q8_prefix(*ref.q8_store(vals))
    want = ref.attend_f64(q, k_used, v_used, ref.causal_mask(n, n, 0, 0), heads, kv)
    scale = np.abs(want).max()
    dk, dv, dq = (torch.from_numpy(a).cuda() for a in (keys, vals, q))
    with att.KVCache(8, 1, kv, hd, cache_type) as full, att.KVCache(8, 1, kv, hd, cache_type) as chunked:
        full.update(0, dk, dv, 0, check=True)
        whole = att.attend(dq, full, 0, n, 0).cpu().numpy()
        assert np.abs(whole - want).max() <= 1e-5 * scale
        for b, e in ((0, 3), (3, 4), (4, 5)):
            chunked.update(0, dk[b:e], dv[b:e], b, check=True)
            part = att.attend(dq[b:e].contiguous(), chunked, 0, e, b).cpu().numpy()
            assert np.abs(part - want[b:e]).max() <= 1e-5 * scale



def test_attention_into_strided_rows(cuda, att):
    """Output rows wider than n_heads * head_dim: the padding stays untouched."""
    torch = cuda
    rng = np.random.default_rng(3)
    count, heads, kv, hd, end = 3, 32, 8, 128, 200
    keys = rng.standard_normal((end, kv, hd)).astype(np.float32)
    vals = rng.standard_normal((end, kv, hd)).astype(np.float32)
    q = rng.standard_normal((count, heads, hd)).astype(np.float32)
    with att.KVCache(256, 1, kv, hd, "f32") as cache:
        cache.update(0, torch.from_numpy(keys).cuda(), torch.from_numpy(vals).cuda(), 0, check=True)
        wide = torch.full((count, heads * hd + 64), 7.0, device="cuda")
        att.attend(torch.from_numpy(q).cuda(), cache, 0, end, end - count, out=wide[:, :heads * hd])
        got = wide.cpu().numpy()
    want = ref.attend_f64(q, keys, vals, ref.causal_mask(count, end, end - count, 0), heads, kv)
    assert np.abs(got[:, :heads * hd] - want).max() <= 1e-5 * np.abs(want).max()
    assert np.all(got[:, heads * hd:] == 7.0)


_TWO_LAUNCH_CHECK = """
import sys
sys.path[:0] = [{root!r}, {root!r} + '/oracle', {root!r} + '/tests']
import importlib
import numpy as np
import torch
import attention as ref
att = importlib.import_module('cl-inference_b200.attention')
for count, heads, kv, hd, end, qstart, kind in [(1, 32, 8, 128, 1000, 999, 'f32'), (6, 64, 8, 128, 70, 64, 'q8'),
                                               (4, 2, 1, 8, 4, 0, 'f32'), (2, 32, 8, 128, 2000, 1998, 'f32'),
                                               (3, 16, 1, 64, 900, 897, 'f32')]:
    rng = np.random.default_rng(end)
    keys = rng.standard_normal((end, kv, hd)).astype(np.float32)
    vals = rng.standard_normal((end, kv, hd)).astype(np.float32)
    q = rng.standard_normal((count, heads, hd)).astype(np.float32)
    with att.KVCache(2048, 1, kv, hd, kind) as cache:
        cache.update(0, torch.from_numpy(keys).cuda(), torch.from_numpy(vals).cuda(), 0, check=True)
        out = att.attend(torch.from_numpy(q).cuda(), cache, 0, end, qstart).cpu().numpy()
    if kind == 'q8':
        keys, vals = ref.q8_prefix(*ref.q8_store(keys)), ref.q8_prefix(*ref.q8_store(vals))
    want = ref.attend_f64(q, keys, vals, ref.causal_mask(count, end, qstart, 0), heads, kv)
    assert np.abs(out - want).max() <= 1e-5 * np.abs(want).max(), (count, end)
print("ok")
"""


def test_vector_staging_of_f32_rows():
    """CLQ_ATTN_BULK=0 stages f32 key and value rows with vector loads instead
    of bulk copies.  A fresh process, since the knob is read once per process."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    proc = subprocess.run([sys.executable, "-c", _TWO_LAUNCH_CHECK.format(root=root)], capture_output=True, text=True,
                          timeout=600, env={**os.environ, "CLQ_ATTN_BULK": "0"})
    assert proc.returncode == 0 and proc.stdout.strip().endswith("ok"), proc.stderr[-3000:]
