"""The benchmark's named shapes at their full sizes, against the fp64 oracle (needs a B200).

Every shape a benchmark workload runs goes through the kernel it takes there:
  * the Llama-3-8B prefill GEMM at a 2048-token prompt (q, gate, the Q6_K down
    projection, and a slice of the 128256-row Q6_K output head);
  * the Llama-3-70B decode linears at one and eight activation rows: q/o
    8192 x 8192, k/v 1024 x 8192, gate/up 28672 x 8192 and the Q6_K down
    projection 8192 x 28672, whose activations do not fit one CTA, so K is
    split across a thread-block cluster;
  * the 128256 x 4096 Q6_K output head at eight and sixty-four rows (at 64
    rows fp32 activations take the exact GEMM, bf16 ones the fp16-operand
    GEMM).
The fp64 check runs on slices of weight rows (start, middle, end) so the
oracle finishes in seconds; the device computes the whole output.  Decode
products meet the reference's bound 1e-5 + 1e-5 * sum|x*w|
(tests/local/packed.lisp:5-12) and the norm-relative gate 1e-3; GEMM
products (fp16 operands) the gate and 1e-3 * sum|x*w|.
"""
import numpy as np
import pytest

from helpers import NORM_REL, element_bound_ok, max_row_relative_error

pytestmark = pytest.mark.gpu


def row_slices(n, rows):
    rows = min(rows, n)
    return sorted({0, (n // 2) // 16 * 16, n - rows})


def check_rows(clq, oracle, dtype, out, x, data, n, k, rows, gemm):
    dt = clq.DTYPES[dtype]
    rb = k // dt.block_size * dt.block_bytes
    for start in row_slices(n, rows):
        cnt = min(rows, n - start)
        ref, mag = oracle.matmul_f64(dtype, x, data[start * rb:(start + cnt) * rb], cnt)
        got = out[:, start:start + cnt]
        assert np.all(np.isfinite(got))
        assert max_row_relative_error(got, ref) <= NORM_REL, (dtype, n, k, start)
        if gemm:
            assert np.all(np.abs(got.astype(np.float64) - ref) <= 1e-3 * mag + 1e-6), (dtype, n, k, start)
        else:
            assert element_bound_ok(got, ref, mag), (dtype, n, k, start)


@pytest.mark.parametrize("dtype,n,k", [
    ("q4_k", 4096, 4096),     # q / o projection
    ("q4_k", 14336, 4096),    # gate / up
    ("q6_k", 4096, 14336),    # down (Q6_K in Q4_K_M)
])
def test_llama3_8b_prefill_2048_tokens(cuda, clq, synth, oracle, dtype, n, k):
    torch = cuda
    m = 2048
    data = synth.packed_blocks(dtype, n, k, seed=5000 + n + k)
    x = torch.from_numpy(synth.activations(m, k, seed=5100)).cuda().to(torch.bfloat16)
    store = clq.Store(dtype, n, k, data)
    out = store.linear(x).cpu().numpy()
    check_rows(clq, oracle, dtype, out, x.float().cpu().numpy(), data, n, k, 192, gemm=True)
    store.close()


def test_llama3_8b_prefill_output_head_slice(cuda, clq, synth, oracle):
    """The last 8256 rows of the Q6_K head (a ragged row count) at 2048 tokens."""
    torch = cuda
    n, k, m = 128256, 4096, 2048
    begin = 120000
    rows = n - begin
    data = synth.packed_blocks("q6_k", n, k, seed=5200)
    x = torch.from_numpy(synth.activations(m, k, seed=5201)).cuda().to(torch.bfloat16)
    store = clq.Store("q6_k", n, k, data)
    out = store.linear(x, row_begin=begin, rows=rows).cpu().numpy()
    rb = k // 256 * 210
    check_rows(clq, oracle, "q6_k", out, x.float().cpu().numpy(), data[begin * rb:], rows, k, 160, gemm=True)
    store.close()


@pytest.mark.parametrize("m", [1, 8])
@pytest.mark.parametrize("dtype,n,k", [
    ("q4_k", 8192, 8192),     # q / o
    ("q4_k", 1024, 8192),     # k / v
    ("q4_k", 28672, 8192),    # gate / up
    ("q6_k", 8192, 28672),    # down: K split across a cluster
])
def test_llama3_70b_decode_linears(cuda, clq, synth, oracle, dtype, n, k, m):
    torch = cuda
    data = synth.packed_blocks(dtype, n, k, seed=6000 + n + k)
    x = synth.activations(m, k, seed=6100 + m)
    store = clq.Store(dtype, n, k, data)
    out = store.linear(torch.from_numpy(x).cuda()).cpu().numpy()
    check_rows(clq, oracle, dtype, out, x, data, n, k, 256, gemm=False)
    again = store.linear(torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), again.view(np.uint32))
    store.close()


@pytest.mark.parametrize("m,xtype", [(8, "float32"), (64, "float32"), (64, "bfloat16")])
def test_q6k_output_head_batched(cuda, clq, synth, oracle, m, xtype):
    torch = cuda
    n, k = 128256, 4096
    data = synth.packed_blocks("q6_k", n, k, seed=7000)
    x = torch.from_numpy(synth.activations(m, k, seed=7001 + m)).cuda().to(getattr(torch, xtype))
    store = clq.Store("q6_k", n, k, data)
    out = store.linear(x).cpu().numpy()
    check_rows(clq, oracle, "q6_k", out, x.float().cpu().numpy(), data, n, k, 256, gemm=xtype != "float32")
    store.close()


@pytest.mark.parametrize("dtype,n,k,m", [
    ("q4_k", 2048, 4096, 512),     # the 256-row Q4_K kernel, a slice of the q/gate rows
    ("q4_k", 1000, 4096, 300),     # ragged rows and tokens
    ("q6_k", 1024, 14336, 256),    # the down projection's format
])
def test_prefill_on_quantized_normal_weights(cuda, clq, synth, oracle, dtype, n, k, m):
    """The prefill configuration's weights: N(0, 0.02) quantized to Q4_K /
    Q6_K.  The GEMM's fp16 operands keep the norm-relative error under 1e-3
    on them too."""
    torch = cuda
    data = getattr(synth, "quantize_" + dtype)(synth.normal_weight(n, k, seed=n + k))
    x = torch.from_numpy(synth.activations(m, k, seed=m)).cuda().to(torch.bfloat16)
    store = clq.Store(dtype, n, k, data)
    out = store.linear(x).cpu().numpy()
    check_rows(clq, oracle, dtype, out, x.float().cpu().numpy(), data, n, k, 128, gemm=True)
    store.close()
