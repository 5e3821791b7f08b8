"""Work fused around the linear (clq_linear_fused_device), needs a B200.

The product's input h is the RMSNorm (local/blocks.lisp:115-116) of x, or the
SwiGLU product silu(gate) * x fed to the down projection (:151-154); the
output may add a residual (layer-forward, :387-392).  The decode GEMV applies
these itself; other shapes (Q4_0 / Q8_0, more activation rows, the prefill
GEMM) run them as separate kernels.  Each case is checked against the fp64
oracle applied to h (formed in fp64 from the same inputs) with the
reference's per-element bound, and the norm-relative gate.
"""
import numpy as np
import pytest

from helpers import NORM_REL, element_bound_ok, max_row_relative_error

pytestmark = pytest.mark.gpu


def silu(g):
    return g / (1.0 + np.exp(-g))


def fused_input(x, gate=None, norm_w=None, eps=1e-5):
    h = x.astype(np.float64)
    if gate is not None:
        h = silu(gate.astype(np.float64)) * h
    if norm_w is not None:
        h = h / np.sqrt(np.mean(h * h, axis=1, keepdims=True) + eps) * norm_w.astype(np.float64)
    return h.astype(np.float32)


def check(got, ref, mag, gemm=False):
    assert max_row_relative_error(got, ref) <= NORM_REL
    if gemm:  # 16-bit operands: tests/test_gpu_gemm.py's bound
        assert np.all(np.abs(got.astype(np.float64) - ref) <= 1e-3 * mag + 1e-6)
    else:
        assert element_bound_ok(got, ref, mag)


@pytest.mark.parametrize("dtype", ["q4_k", "q6_k", "q4_0", "q8_0"])
@pytest.mark.parametrize("m", [1, 2, 5])
def test_rmsnorm_prologue(cuda, clq, synth, oracle, dtype, m):
    torch = cuda
    n, k = 300, 2048
    data = synth.packed_blocks(dtype, n, k, seed=11)
    rng = np.random.default_rng(m)
    x = (rng.standard_normal((m, k)) * 3).astype(np.float32)
    w = (rng.standard_normal(k) * 0.5 + 1).astype(np.float32)
    store = clq.Store(dtype, n, k, data)
    got = clq.linear_fused(store, torch.from_numpy(x).cuda(), norm_weight=torch.from_numpy(w).cuda(),
                           eps=1e-6).cpu().numpy()
    ref, mag = oracle.matmul_f64(dtype, fused_input(x, norm_w=w, eps=1e-6), data, n)
    check(got, ref, mag)
    store.close()


@pytest.mark.parametrize("dtype", ["q4_k", "q6_k", "q4_0"])
@pytest.mark.parametrize("m", [1, 2, 5])
def test_swiglu_prologue_and_residual(cuda, clq, synth, oracle, dtype, m):
    torch = cuda
    n, k = 257, 1024
    data = synth.packed_blocks(dtype, n, k, seed=12)
    rng = np.random.default_rng(10 + m)
    up = rng.standard_normal((m, k)).astype(np.float32)
    gate = (rng.standard_normal((m, k)) * 4).astype(np.float32)
    res = rng.standard_normal((m, n)).astype(np.float32)
    store = clq.Store(dtype, n, k, data)
    out = torch.from_numpy(res).cuda()  # in place: out is the residual stream
    clq.linear_fused(store, torch.from_numpy(up).cuda(), out=out, gate=torch.from_numpy(gate).cuda(), residual=out)
    ref, mag = oracle.matmul_f64(dtype, fused_input(up, gate=gate), data, n)
    check(out.cpu().numpy(), ref + res.astype(np.float64), mag + np.abs(res))
    store.close()


@pytest.mark.parametrize("xtype", ["float32", "bfloat16"])
def test_grouped_projections_share_one_normalized_input(cuda, clq, synth, oracle, xtype):
    torch = cuda
    k = 4096
    shapes = [4096, 1024, 1024]
    datas = [synth.packed_blocks("q4_k", n, k, seed=20 + i) for i, n in enumerate(shapes)]
    stores = [clq.Store("q4_k", n, k, d) for n, d in zip(shapes, datas)]
    rng = np.random.default_rng(3)
    w = (rng.standard_normal(k) * 0.3 + 1).astype(np.float32)
    for m in (1, 2):
        x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda().to(getattr(torch, xtype))
        outs = clq.linear_group_fused(stores, x, norm_weight=torch.from_numpy(w).cuda(), eps=1e-5)
        h = fused_input(x.float().cpu().numpy(), norm_w=w, eps=1e-5)
        for o, d, n, s in zip(outs, datas, shapes, stores):
            ref, mag = oracle.matmul_f64("q4_k", h, d, n)
            check(o.cpu().numpy(), ref, mag)
            # one launch per member partitions the tiles differently (its K
            # split between warps rounds differently): both meet the bound
            single = clq.linear_fused(s, x, norm_weight=torch.from_numpy(w).cuda(), eps=1e-5)
            check(single.cpu().numpy(), ref, mag)
    for s in stores:
        s.close()


def test_prefill_gemm_takes_the_fusion_as_separate_kernels(cuda, clq, synth, oracle):
    torch = cuda
    n, k, m = 512, 1024, 64
    data = synth.packed_blocks("q4_k", n, k, seed=30)
    rng = np.random.default_rng(4)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda().to(torch.bfloat16)
    w = (rng.standard_normal(k) * 0.2 + 1).astype(np.float32)
    res = torch.from_numpy(rng.standard_normal((m, n)).astype(np.float32)).cuda()
    store = clq.Store("q4_k", n, k, data)
    got = clq.linear_fused(store, x, norm_weight=torch.from_numpy(w).cuda(), residual=res).cpu().numpy()
    h = fused_input(x.float().cpu().numpy(), norm_w=w)
    ref, mag = oracle.matmul_f64("q4_k", h, data, n)
    r = res.cpu().numpy().astype(np.float64)
    check(got, ref + r, mag + np.abs(r), gemm=True)
    store.close()


def test_fusion_argument_checks(cuda, clq, synth):
    torch = cuda
    data = synth.packed_blocks("q4_k", 16, 256, seed=1)
    store = clq.Store("q4_k", 16, 256, data)
    x = torch.zeros(1, 256, device="cuda")
    with pytest.raises(ValueError):
        clq.linear_fused(store, x, norm_weight=torch.ones(255, device="cuda"))
    with pytest.raises(clq.ClqError):
        clq.linear_fused(store, x, norm_weight=torch.ones(256, device="cuda"), eps=-1.0)
    with pytest.raises(clq.ClqError):
        clq.linear_fused(store, x, residual=torch.zeros(1, 8, device="cuda"))
    store.close()
