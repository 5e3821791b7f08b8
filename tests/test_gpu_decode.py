"""Decode products of one to eight activation rows on Q4_K, Q6_K, Q4_0 and Q8_0
(needs a B200).

These shapes run the per-warp streaming GEMV: every warp copies its own
(16-row, 256-column) units with a tensor-map box and the tile partials meet
through a per-tile count in shared memory.  Where the activations of all of K
do not fit in a CTA's shared memory (several rows, long rows) K is split
between the CTAs of a thread-block cluster, each of which reads the others'
tile sums through distributed shared memory and adds them in split order:
results are still the same bits on every call, also when calls of other
shapes run in between.  Cases cover ragged row counts
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
@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
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


@pytest.mark.parametrize("dtype", ["q4_0", "q8_0"])
@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("n,k", [(300, 2048), (1000, 4096), (77, 14336)])
def test_q4_0_q8_0_decode_rows_against_oracle(cuda, clq, synth, oracle, dtype, m, n, k):
    """Q4_0 / Q8_0 rows of at least 4096, or eight activation rows, stream
    through the per-warp kernel (swizzled 16-row units, one s8 or u8 MMA per
    32-element block); shorter rows at one to four tokens take the
    register-fed kernel.  Both meet the reference's bound, bit-stable."""
    torch = cuda
    data = synth.packed_blocks(dtype, n, k, seed=3 * n + k + m)
    for xtype in ("float32", "bfloat16"):
        x = torch.from_numpy(synth.activations(m, k, seed=5 * m + k)).cuda().to(getattr(torch, xtype))
        store = clq.Store(dtype, n, k, data)
        got = store.linear(x).cpu().numpy()
        ref, mag = oracle.matmul_f64(dtype, x.float().cpu().numpy(), data, n)
        check(got, ref, mag)
        again = store.linear(x).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
        store.close()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("xtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("m", [1, 2, 4, 7])
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
    for scales in ((1e-30, 1e30), (0.0, 1e4), (1e4, 1e-30, 0.0, 1e30, 1.0, 1e-3)):
        x = rng.standard_normal((len(scales), k)).astype(np.float32)
        for i, sc in enumerate(scales):
            x[i] *= np.float32(sc)
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
    for m in (1, 2, 4, 8):
        x = synth.activations(m, k, seed=95 + m)
        outs = clq.linear_group(stores, torch.from_numpy(x).cuda())
        for o, d, n in zip(outs, datas, shapes):
            ref, mag = oracle.matmul_f64(dtype, x, d, n)
            check(o.cpu().numpy(), ref, mag)
    for s in stores:
        s.close()


@pytest.mark.parametrize("dtype", DTYPES)
def test_split_k_calls_of_other_shapes_in_between(cuda, clq, synth, oracle, dtype):
    """K-split launches of different tile counts and split counts, in turn:
    each tile's count must be back at zero after every call."""
    torch = cuda
    cases = [(2000, 4096, 8), (77, 14336, 5), (4100, 1024, 6), (515, 14336, 3)]
    runs = []
    for i, (n, k, m) in enumerate(cases):
        data = synth.packed_blocks(dtype, n, k, seed=300 + i)
        x = torch.from_numpy(synth.activations(m, k, seed=310 + i)).cuda()
        runs.append((clq.Store(dtype, n, k, data), x, data, n))
    first = [s.linear(x).cpu().numpy() for s, x, _, _ in runs]
    for (s, x, data, n), got in zip(runs, first):
        ref, mag = oracle.matmul_f64(dtype, x.cpu().numpy(), data, n)
        check(got, ref, mag)
    for _ in range(2):
        for (s, x, _, _), want in zip(reversed(runs), reversed(first)):
            again = s.linear(x).cpu().numpy()
            assert np.array_equal(again.view(np.uint32), want.view(np.uint32))
    for s, *_ in runs:
        s.close()
