"""Decode products of one and two activation rows on Q4_K and Q6_K (needs a B200).

These shapes run the per-warp streaming GEMV: every warp copies its own
(16-row, 256-column) units with a tensor-map box and the tile partials meet
through a per-tile count in shared memory.  Cases cover ragged row counts
(boxes that run past the last row read zeros), row views written into a wider
output, K from one superblock to a 14336-wide down projection, the three
activation types, an activation pointer off the 16-byte grid, and activations
spanning the fp32 range.  The bound is the reference's per-element one
(tests/local/packed.lisp:5-12) and the norm-relative gate.
"""
import numpy as np
import pytest

from helpers import NORM_REL, element_bound_ok, max_row_relative_error

pytestmark = pytest.mark.gpu
DTYPES = ["q4_k", "q6_k"]


def check(got, ref, mag):
    assert max_row_relative_error(got, ref) <= NORM_REL
    assert element_bound_ok(got, ref, mag)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("n,k", [(300, 2048), (77, 14336), (4100, 256), (2000, 4096)])
def test_decode_rows_against_oracle(cuda, clq, synth, oracle, dtype, m, n, k):
    torch = cuda
    data = synth.packed_blocks(dtype, n, k, seed=n + k + m)
    x = synth.activations(m, k, seed=7 * m + k)
    store = clq.Store(dtype, n, k, data)
    got = store.linear(torch.from_numpy(x).cuda()).cpu().numpy()
    ref, mag = oracle.matmul_f64(dtype, x, data, n)
    check(got, ref, mag)
    # the same launch twice gives the same bits
    again = store.linear(torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
    store.close()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("xtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("m", [1, 2])
def test_decode_views_types_and_unaligned_activations(cuda, clq, synth, oracle, dtype, xtype, m):
    torch = cuda
    n, k = 333, 1024
    data = synth.packed_blocks(dtype, n, k, seed=41 + m)
    # activations one element past a 16-byte boundary
    flat = torch.zeros(m * k + 1, dtype=getattr(torch, xtype), device="cuda")
    flat[1:] = torch.from_numpy(synth.activations(m, k, seed=42 + m).reshape(-1)).cuda().to(flat.dtype)
    x = flat[1:].view(m, k)
    assert x.data_ptr() % 16 != 0
    ref, mag = oracle.matmul_f64(dtype, x.float().cpu().numpy(), data, n)
    store = clq.Store(dtype, n, k, data)
    out = torch.full((m, n + 5), float("nan"), device="cuda")
    for begin, rows in ((0, 17), (17, 160), (177, 156)):
        store.linear(x, out=out[:, begin:begin + rows], row_begin=begin, rows=rows)
    assert torch.isnan(out[:, n:]).all()
    check(out[:, :n].cpu().numpy(), ref, mag)
    store.close()


@pytest.mark.parametrize("dtype", DTYPES)
def test_decode_extreme_activation_scales(cuda, clq, synth, oracle, dtype):
    torch = cuda
    n, k = 64, 4096
    data = synth.packed_blocks(dtype, n, k, seed=9)
    rng = np.random.default_rng(3)
    store = clq.Store(dtype, n, k, data)
    for scale_a, scale_b in ((1e-30, 1e30), (0.0, 1e4)):
        x = rng.standard_normal((2, k)).astype(np.float32)
        x[0] *= np.float32(scale_a)
        x[1] *= np.float32(scale_b)
        x[1, ::5] = 0.0
        ref, mag = oracle.matmul_f64(dtype, x, data, n)
        got = store.linear(torch.from_numpy(x).cuda()).cpu().numpy().astype(np.float64)
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - ref) <= 1e-5 * mag + 1e-37)
    store.close()


@pytest.mark.parametrize("dtype", DTYPES)
def test_decode_group_of_projections(cuda, clq, synth, oracle, dtype):
    """q/k/v-shaped members in one launch, ragged and tile-aligned row counts."""
    torch = cuda
    k = 4096
    shapes = [4096, 1024, 1000]
    datas = [synth.packed_blocks(dtype, n, k, seed=90 + i) for i, n in enumerate(shapes)]
    stores = [clq.Store(dtype, n, k, d) for n, d in zip(shapes, datas)]
    for m in (1, 2):
        x = synth.activations(m, k, seed=95 + m)
        outs = clq.linear_group(stores, torch.from_numpy(x).cuda())
        for o, d, n in zip(outs, datas, shapes):
            ref, mag = oracle.matmul_f64(dtype, x, d, n)
            check(o.cpu().numpy(), ref, mag)
    for s in stores:
        s.close()
