"""The tensor-core prefill GEMM (tcgen05) against the fp64 oracle (needs a B200).

Taken for many activation rows (prompt tokens) with 16-bit activations, or
with CLQ_MATH_FAST for fp32 ones.  Its operands are fp16 (each dequantized
weight and each power-of-two-scaled activation rounded once), so the gate is
the linear-output tolerance -- max over rows of ||y - y64|| / ||y64|| <= 1e-3 --
plus a per-element bound of 1e-3 * sum|x*w| for the two fp16 roundings.
"""
import numpy as np
import pytest

from helpers import NORM_REL, max_row_relative_error

pytestmark = pytest.mark.gpu
FAST = 1


def check(out, ref, mag):
    assert np.all(np.isfinite(out))
    assert max_row_relative_error(out, ref) <= NORM_REL
    assert np.all(np.abs(out.astype(np.float64) - ref) <= 1e-3 * mag + 1e-6)


@pytest.mark.parametrize("dtype", ["q4_k", "q6_k", "q4_0", "q8_0"])
@pytest.mark.parametrize("n,k,m", [(200, 512, 64), (128, 1024, 100), (384, 768, 300)])
def test_gemm_small_shapes(cuda, clq, synth, oracle, dtype, n, k, m):
    torch = cuda
    data = synth.packed_blocks(dtype, n, k, seed=n + k + m)
    x = torch.from_numpy(synth.activations(m, k, seed=m)).cuda().to(torch.bfloat16)
    store = clq.Store(dtype, n, k, data)
    out = store.linear(x).cpu().numpy()
    ref, mag = oracle.matmul_f64(dtype, x.float().cpu().numpy(), data, n)
    check(out, ref, mag)
    store.close()


@pytest.mark.parametrize("xtype", ["float16", "float32"])
def test_gemm_activation_types(cuda, clq, synth, oracle, xtype):
    torch = cuda
    n, k, m = 256, 1024, 128
    data = synth.packed_blocks("q4_k", n, k, seed=7)
    x = torch.from_numpy(synth.activations(m, k, seed=8)).cuda().to(getattr(torch, xtype))
    store = clq.Store("q4_k", n, k, data)
    out = store.linear(x, flags=FAST).cpu().numpy()
    ref, mag = oracle.matmul_f64("q4_k", x.float().cpu().numpy(), data, n)
    check(out, ref, mag)
    store.close()


def test_gemm_extreme_activation_magnitudes(cuda, clq, synth, oracle):
    """Per-token power-of-two scaling keeps tiny and huge rows in fp16 range."""
    torch = cuda
    n, k, m = 256, 1024, 64
    data = synth.packed_blocks("q6_k", n, k, seed=9)
    x = synth.activations(m, k, seed=10)
    x[0] *= np.float32(1e-20)
    x[1] *= np.float32(1e20)
    x[2] = 0.0
    store = clq.Store("q6_k", n, k, data)
    out = store.linear(torch.from_numpy(x).cuda(), flags=FAST).cpu().numpy().astype(np.float64)
    ref, mag = oracle.matmul_f64("q6_k", x, data, n)
    assert np.all(np.isfinite(out))
    assert np.all(np.abs(out - ref) <= 1e-3 * mag + 1e-30)
    store.close()


@pytest.mark.parametrize("dtype,n,k,m", [
    ("q4_k", 4096, 4096, 512),    # Llama-3-8B q/o projection, 512-token prompt
    ("q4_k", 14336, 4096, 128),   # gate/up, 128-token prompt
    ("q6_k", 4096, 14336, 256),   # down projection (Q6_K in Q4_K_M)
])
def test_gemm_prefill_shapes(cuda, clq, synth, oracle, dtype, n, k, m):
    torch = cuda
    data = synth.packed_blocks(dtype, n, k, seed=4000 + n)
    x = torch.from_numpy(synth.activations(m, k, seed=4100 + m)).cuda().to(torch.bfloat16)
    store = clq.Store(dtype, n, k, data)
    out = store.linear(x).cpu().numpy()
    rows = 384  # fp64 check on a slice of weight rows at the start, middle and end
    rb = k // clq.DTYPES[dtype].block_size * clq.DTYPES[dtype].block_bytes
    xf = x.float().cpu().numpy()
    for start in (0, n // 2, n - rows):
        ref, mag = oracle.matmul_f64(dtype, xf, data[start * rb:(start + rows) * rb], rows)
        check(out[:, start:start + rows], ref, mag)
    store.close()


def test_gemm_repeats_bit_identically(cuda, clq, synth):
    torch = cuda
    n, k, m = 512, 2048, 200
    data = synth.packed_blocks("q4_k", n, k, seed=11)
    x = torch.from_numpy(synth.activations(m, k, seed=12)).cuda().to(torch.bfloat16)
    store = clq.Store("q4_k", n, k, data)
    a = store.linear(x)
    b = store.linear(x)
    assert torch.equal(a, b)
    store.close()


_MODE_CHECK = r"""
import sys
sys.path[:0] = [{root!r}, {root!r} + "/oracle", {root!r} + "/tests"]
import importlib
import numpy as np
import torch
import oracle
from helpers import NORM_REL, max_row_relative_error
clq = importlib.import_module("cl-inference_b200")
synth = importlib.import_module("cl-inference_b200.synth")
torch.cuda.set_device(0)
for n, k, m in ((2048, 4096, 512), (1000, 1024, 300), (300, 2048, 96)):
    data = synth.quantize_q4_k(synth.normal_weight(n, k, seed=n + m))
    x = torch.from_numpy(synth.activations(m, k, seed=m)).cuda().to(torch.bfloat16)
    store = clq.Store("q4_k", n, k, data)
    out = store.linear(x).cpu().numpy().astype(np.float64)
    rb = k // 256 * 144
    for start in sorted({{0, n - 128}}):
        ref, mag = oracle.matmul_f64("q4_k", x.float().cpu().numpy(), data[start * rb:(start + 128) * rb], 128)
        got = out[:, start:start + 128]
        assert max_row_relative_error(got, ref) <= NORM_REL, (n, k, m, start)
        assert np.all(np.abs(got - ref) <= 1e-3 * mag + 1e-6), (n, k, m, start)
    store.close()
print("ok")
"""


@pytest.mark.parametrize("mode", ["1", "2"])
def test_256_row_q4k_kernels(mode):
    """The 256-row Q4_K kernel in both forms (CLQ_GEMM_TMA=1: packed
    superblocks staged by tensor-map copies; 2: register-fed), against the
    fp64 oracle on N(0, 0.02) weights; a fresh process, since the knob is read
    once per process."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    proc = subprocess.run([sys.executable, "-c", _MODE_CHECK.format(root=root)], capture_output=True, text=True,
                          timeout=600, env={**os.environ, "CLQ_GEMM_TMA": mode})
    assert proc.returncode == 0 and proc.stdout.strip().endswith("ok"), proc.stderr[-3000:]


@pytest.mark.parametrize("dtype", ["q4_k", "q6_k", "q4_0", "q8_0"])
@pytest.mark.parametrize("n,k,m", [(300, 1024, 64), (1024, 4096, 200)])
def test_exact_gemm_meets_the_reference_bound(cuda, clq, synth, oracle, dtype, n, k, m):
    """fp32 activations with default flags take the exact GEMM (weights and
    activations split into fp16 hi + scaled lo parts, a second accumulator
    for the cross terms): the reference's own bound 1e-5 + 1e-5 * sum|x*w|
    (tests/local/packed.lisp:5-12), on uniform codes and on N(0, 0.02)
    weights quantized to the K formats."""
    torch = cuda
    if dtype in ("q4_k", "q6_k"):
        data = getattr(synth, "quantize_" + dtype)(synth.normal_weight(n, k, seed=n + k))
    else:
        data = synth.packed_blocks(dtype, n, k, seed=n + k + m)
    x = synth.activations(m, k, seed=m + 1)
    x[0] *= np.float32(1e-20)
    x[1] *= np.float32(1e20)
    store = clq.Store(dtype, n, k, data)
    out = store.linear(torch.from_numpy(x).cuda()).cpu().numpy().astype(np.float64)
    ref, mag = oracle.matmul_f64(dtype, x, data, n)
    assert np.all(np.isfinite(out))
    assert np.all(np.abs(out - ref) <= 1e-5 * mag + 1e-37), np.max(np.abs(out - ref) / (mag + 1e-37))
    # bf16 activations with CLQ_MATH_EXACT take the same form
    xb = torch.from_numpy(x[2:]).cuda().to(torch.bfloat16)
    outb = store.linear(xb, flags=4).cpu().numpy().astype(np.float64)
    refb, magb = oracle.matmul_f64(dtype, xb.float().cpu().numpy(), data, n)
    assert np.all(np.abs(outb - refb) <= 1e-5 * magb + 1e-37)
    store.close()


@pytest.mark.parametrize("dtype,m,xtype", [("q4_k", 128, "bfloat16"), ("q6_k", 64, "float32"), ("q4_0", 40, "float32")])
def test_grouped_gemm_shares_one_activation_image(cuda, clq, synth, oracle, dtype, m, xtype):
    """A group (q/k/v shapes) through the GEMM forms the activation image once
    and gives each member the bits of its own call."""
    torch = cuda
    k = 2048
    shapes = [512, 128, 300]
    datas = [synth.packed_blocks(dtype, n, k, seed=70 + i) for i, n in enumerate(shapes)]
    stores = [clq.Store(dtype, n, k, d) for n, d in zip(shapes, datas)]
    x = torch.from_numpy(synth.activations(m, k, seed=m)).cuda().to(getattr(torch, xtype))
    outs = clq.linear_group(stores, x)
    xf = x.float().cpu().numpy()
    for st, d, n, o in zip(stores, datas, shapes, outs):
        single = st.linear(x).cpu().numpy()
        got = o.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), single.view(np.uint32))
        ref, mag = oracle.matmul_f64(dtype, xf, d, n)
        bound = 1e-5 if xtype == "float32" else 1e-3
        assert np.all(np.abs(got.astype(np.float64) - ref) <= bound * mag + 1e-6)
    for st in stores:
        st.close()
