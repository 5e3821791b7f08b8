#!/usr/bin/env python
"""Benchmark: the packed linears of one decode step of a Llama-3-8B-shaped Q4_K-M model.

A step is every quantized linear of one token (M = 1): 32 layers x (q, k, v, o,
gate, up in Q4_K; down in Q6_K) plus the Q6_K output head, 4.84 GB of packed
weights -- far larger than the 126 MB L2, so no flush is needed between steps.
At N GPUs the linears are tensor-parallel (column-parallel q/k/v/gate/up/head,
row-parallel o/down, two all-reduces per layer and an all-gather of the logits).

Prints one JSON line (rank 0): whole-job HBM GB/s over the step, tok/s, the
roofline of the dominant kernel (the Q4_K GEMV), the CPU baseline, the
end-to-end number through the host-buffer C ABI, and clocks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl clq|reference]
"""
import argparse
import datetime
import importlib
import json
import os
import pathlib
import statistics
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "oracle"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "quant GEMV HBM GB/s (%peak) + 8B-shape Q4_K decode tok/s @1/2/4/8 GPU"
FALLBACK_HBM_GBS = 6650.0

# GEMV sweeps (one GPU): (dtype, out rows, in columns) per shape.  A step runs
# every shape once over distinct weight copies, enough copies that the step's
# weights exceed four times the 126 MB L2.
SWEEPS = {
    "q8_0-4096": [("q8_0", 4096, 4096)],
    "q4-llama32-1b": [(d, n, k) for d in ("q4_0", "q4_k")
                      for n, k in ((2048, 2048), (512, 2048), (8192, 2048), (8192, 2048), (2048, 8192))],
    "q6k-vocab-qwen3-8b": [("q6_k", 128256, 4096)] + [("q6_k", n, k) for n, k in
                           ((4096, 4096), (1024, 4096), (1024, 4096), (12288, 4096), (12288, 4096), (4096, 12288))],
}


def workload_linears(args, tp, cfg):
    """(name, dtype, n, k, tp kind, input buffer) of one step of the workload."""
    if args.workload == "step":
        return tp.model_linears(cfg)
    shapes = SWEEPS[args.workload]
    once = sum(tp.weight_bytes(d, n, k) for d, n, k in shapes)
    copies = max(1, -(-4 * 126 * 2**20 // once))
    return [(f"{d}.{n}x{k}.{c}.{i}", d, n, k, "rows", f"k{k}")
            for c in range(copies) for i, (d, n, k) in enumerate(shapes)]
FALLBACK_BF16_TFLOPS = 1590.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["clq", "reference"], default="clq")
    ap.add_argument("--model", choices=["8b", "70b"], default="8b")
    ap.add_argument("--workload", choices=["step"] + sorted(SWEEPS), default="step",
                    help="step: every linear of one decode step of --model (the headline); "
                         "q8_0-4096 / q4-llama32-1b / q6k-vocab-qwen3-8b: GEMV sweeps over those shapes")
    ap.add_argument("--m", type=int, default=1, help="activation rows (tokens) per step")
    ap.add_argument("--xtype", choices=["f32", "bf16", "f16"], default=None,
                    help="activation type; default f32 for decode (M < 64), bf16 for prefill")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder layers per step (default: the model's); fewer for profiling captures")
    ap.add_argument("--allreduce", choices=["fused", "nccl"], default="fused",
                    help="tensor parallel: row-parallel linears all-reduce inside the GEMV over NVLink "
                         "(fused) or through NCCL after it")
    ap.add_argument("--fusions", choices=["off", "fused", "unfused"], default="off",
                    help="run each layer with the reference's data flow around the linears (RMSNorm -> q/k/v, "
                         "o + residual, RMSNorm -> gate/up, SwiGLU -> down + residual; attention with --attention): "
                         "fused into "
                         "the GEMVs (clq_linear_fused_device), or as torch element-wise ops between plain linears")
    ap.add_argument("--attention", choices=["off", "f32", "q8"], default="off",
                    help="with --fusions: each layer also runs RoPE on q and k, stores k and v in a KV cache of "
                         "that type and attends over --context cached positions (local/blocks.lisp:327-353)")
    ap.add_argument("--context", type=int, default=1024, help="cached positions attended over (with --attention)")
    ap.add_argument("--weights", choices=["auto", "quantized", "uniform"], default="auto",
                    help="quantized: N(0, 0.02) weights quantized to Q4_K / Q6_K on the device; uniform: uniform "
                         "codes and random scales; auto: quantized for decoder steps, uniform for GEMV sweeps")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the named workloads measured after the headline step")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler(threading.Thread):
    """SM clock and throttle reasons through NVML every 10 ms (reads only)."""

    REASONS = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, index):
        super().__init__(daemon=True)
        self.samples, self.reasons, self.stop_flag = [], set(), threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def run(self):
        while self.nv and not self.stop_flag.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                break
            time.sleep(0.01)

    def result(self):
        self.stop_flag.set()
        self.join(timeout=1)
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def peak_tflops():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        try:
            v = json.loads(f.read_text()).get("bf16_tflops")
            if v:
                return float(v), "measured"
        except (ValueError, OSError):
            pass
    return FALLBACK_BF16_TFLOPS, "fallback"


def count_kernel_nodes(graph):
    """(our kernels, all kernels) among the kernel nodes of a captured graph;
    ours are the functions whose name carries the clq namespace."""
    from cuda.bindings import driver as cu
    g = cu.CUgraph(graph.raw_cuda_graph())
    _, _, n = cu.cuGraphGetNodes(g, 0)
    _, nodes, n = cu.cuGraphGetNodes(g, n)
    ours = total = 0
    for node in nodes[:n]:
        _, kind = cu.cuGraphNodeGetType(node)
        if kind != cu.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
            continue
        total += 1
        _, prm = cu.cuGraphKernelNodeGetParams(node)
        name = b""
        if int(prm.func):
            _, name = cu.cuFuncGetName(prm.func)
        elif int(prm.kern):
            _, name = cu.cuKernelGetName(prm.kern)
        if name and b"clq" in name:
            ours += 1
    return ours, total


def dist_setup(torch):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
    return rank, world, local


def device_weight(torch, dtype, n, k, seed):
    """Packed bytes with the configuration's distributions, generated on the device."""
    clq = importlib.import_module("cl-inference_b200")
    dt = clq.find_dtype(dtype)
    nblocks = n * (k // dt.block_size)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    raw = torch.randint(0, 256, (nblocks, dt.block_bytes), dtype=torch.uint8, device="cuda", generator=g)

    def halves(scale):
        v = (torch.randn(nblocks, device="cuda", generator=g).abs() * scale).half()
        return v.view(torch.uint8).view(nblocks, 2)

    if dt.name == "q4_k":
        raw[:, 0:2] = halves(0.01)
        raw[:, 2:4] = halves(0.01)
    elif dt.name == "q6_k":
        raw[:, 192:208] = torch.randint(-64, 64, (nblocks, 16), device="cuda", generator=g).to(torch.int8).view(torch.uint8)
        raw[:, 208:210] = halves(0.005)
    elif dt.name == "q4_0":
        raw[:, 0:2] = halves(0.02 / 8)
    elif dt.name == "q8_0":
        raw[:, 0:2] = halves(0.02 / 127)
        raw[:, 2:34] = torch.randint(-127, 128, (nblocks, 32), device="cuda", generator=g).to(torch.int8).view(torch.uint8)
    return raw.reshape(-1)


# Named workloads measured after the headline (one GPU: every shape list the
# benchmark configurations name; several GPUs: the 70B step tensor-parallel).
# Each is a bounded run: at most 30 timed steps after 3 warm-up steps.
def config_runs(world):
    if world > 1:
        return [(f"c5_llama3_70b_decode_m{m}", dict(model="70b", m=m)) for m in (1, 8)]
    runs = [("c1_q8_0_4096_m1", dict(workload="q8_0-4096", m=1))]
    runs += [(f"c2_llama32_1b_q4_m{m}", dict(workload="q4-llama32-1b", m=m)) for m in (1, 4, 16)]
    runs += [(f"c3_q6k_vocab_qwen3_8b_m{m}", dict(workload="q6k-vocab-qwen3-8b", m=m)) for m in (1, 8, 64)]
    runs += [(f"c4_llama3_8b_prefill_m{m}", dict(m=m)) for m in (128, 512, 2048)]
    # the drop-in prefill: fp32 activations through the exact GEMM (fp32-class products)
    runs += [("c4_llama3_8b_prefill_m512_f32_exact", dict(m=512, xtype="f32"))]
    runs += [(f"c5_llama3_70b_decode_m{m}", dict(model="70b", m=m)) for m in (1, 8)]
    runs += [("llama3_8b_decode_m8", dict(m=8))]
    return runs


def weights_kind(args):
    """The decoder steps use N(0, 0.02) weights quantized to Q4_K / Q6_K (the
    prefill and 70B configurations' recipe); the GEMV sweeps the uniform codes
    their configurations name."""
    if args.weights != "auto":
        return args.weights
    return "quantized" if args.workload == "step" else "uniform"


def device_quantized_weight(torch, dtype, n, k, seed):
    """N(0, 0.02) weights drawn and quantized on the device (synth.py's
    quantizers, the torch form), in row chunks to bound the temporaries."""
    synth = importlib.import_module("cl-inference_b200.synth")
    quant = {"q4_k": synth.quantize_q4_k_torch, "q6_k": synth.quantize_q6_k_torch}.get(dtype)
    if quant is None:
        return device_weight(torch, dtype, n, k, seed)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    parts, step = [], max(1, (1 << 26) // k)
    for r0 in range(0, n, step):
        rows = min(step, n - r0)
        w = torch.randn(rows, k, device="cuda", generator=g) * 0.02
        parts.append(quant(w))
        del w
    return torch.cat(parts)


def run_clq(args):
    import gc

    import torch
    rank, world, local = dist_setup(torch)
    dist = torch.distributed if world > 1 else None
    result = measure(args, torch, rank, world, local, dist)
    headline = (args.workload == "step" and args.model == "8b" and args.m == 1 and args.fusions == "off"
                and args.layers is None and args.xtype is None)
    if headline and not args.no_configs:
        subs = {}
        for name, over in config_runs(world):
            sub = argparse.Namespace(**vars(args))
            sub.workload, sub.model = "step", "8b"
            for key, val in over.items():
                setattr(sub, key, val)
            sub.steps, sub.warmup = min(args.steps, 30), max(3, min(args.warmup, 5))
            sub.no_e2e = sub.no_cpu = True
            gc.collect()
            torch.cuda.empty_cache()
            r = measure(sub, torch, rank, world, local, dist)
            if rank == 0:
                subs[name] = summary(r)
        if rank == 0:
            result["workloads"] = subs
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def summary(r):
    """The compact form of a named workload's line."""
    keep = ("value", "unit", "ms_per_step", "tok_per_s", "tflops", "steps", "gpu_launches_per_step", "check")
    out = {key: r[key] for key in keep if key in r}
    out["workload"] = r["config"]["workload"]
    rf = r.get("roofline") or {}
    out["roofline"] = {key: rf.get(key) for key in ("bound", "kernel", "achieved", "peak", "unit", "frac",
                                                    "us_per_launch")}
    out["clocks"] = {key: r["clocks"].get(key) for key in ("sm_mhz", "reasons")}
    return out


def check_outputs(torch, stores, outs, inputs, m, gemm, world, wide=False):
    """Per-run correctness: sampled output columns against float64 products.

    The reference product is x . dequant(W)^T in float64, with dequant(W) from
    the store's bit-exact dequantize kernel (clq_dequantize_device, the
    reference's element formulas, bit-checked by the tests), for the first and
    last 16 rows (128 for the GEMM) of each checked linear.  Reported as the maximum over
    activation rows of ||y - y64|| / ||y64|| (the reference's metric,
    tests/acceptance/helpers.lisp:153-154) and whether every element meets the
    per-element bound: 1e-5 + 1e-5 * sum|x*w| for the GEMV
    (tests/local/packed.lisp:5-12), 1e-3 * sum|x*w| + 1e-6 for the GEMM's fp16
    operands.  Under tensor parallelism only column-parallel shards are
    checked (a row-parallel output is a sum over ranks)."""
    import numpy as np
    worst, ok, checked = 0.0, True, 0
    rel_tol, abs_tol = (1e-3, 1e-6) if gemm else (1e-5, 1e-5)
    picks = range(len(stores))
    if wide:  # the first decoder layer and the head: the fp64 products grow with M
        picks = list(range(min(7, len(stores)))) + [len(stores) - 1]
    for i in picks:
        store, s, dtype, kind, src, name = stores[i]
        if world > 1 and kind != "rows":
            continue
        x = inputs[src].float().cpu().numpy().astype(np.float64)
        # the norm over a row needs enough columns to be a stable estimate:
        # 16 per end for the GEMV's fp32-class products, 128 for the GEMM's
        per_end = 128 if wide else 16
        for r0 in sorted({0, max(0, s.n - per_end)}):
            cnt = min(per_end, s.n - r0)
            w = store.dequantize(r0, cnt).cpu().numpy().astype(np.float64)
            ref = x @ w.T
            mag = np.abs(x) @ np.abs(w).T
            got = outs[i][:, r0:r0 + cnt].cpu().numpy().astype(np.float64)
            num = np.linalg.norm(got - ref, axis=-1)
            den = np.maximum(np.linalg.norm(ref, axis=-1), 1e-300)
            worst = max(worst, float(np.max(num / den)))
            ok = ok and bool(np.all(np.abs(got - ref) <= abs_tol + rel_tol * mag))
        checked += 1
    return {"max_rel_err": worst, "gate": 1e-3, "element_bound": f"{abs_tol:g} + {rel_tol:g}*sum|x*w|",
            "element_bound_ok": ok, "passed": ok and worst <= 1e-3, "linears_checked": checked,
            "rows_per_linear": 256 if wide else 32,
            "reference": "float64 x . dequant(W)^T, dequant by the store's bit-exact dequantize kernel"}


def config_dict(args, cfg, m, xtype, prefill, world, fuse_mode, job_bytes, n_linears):
    """The line's "config": the workload by name and sizes (shared by both arms)."""
    if args.workload == "step":
        workload = (f"llama3-{args.model}-shape Q4_K-M {'prefill' if prefill else 'decode'} linears, "
                    f"M={m}, {xtype} activations: {cfg['layers']} layers x (q,k,v,o,gate,up Q4_K; "
                    f"down Q6_K) + Q6_K output")
    else:
        shapes = SWEEPS[args.workload]
        workload = (f"GEMV sweep {args.workload}: " + ", ".join(f"{d} {n}x{k}" for d, n, k in shapes)
                    + f"; M={m}, {xtype} activations; {n_linears // len(shapes)} weight copies")
    return {
        "workload": workload, "m": m, "xtype": xtype, "layers": cfg["layers"], "parallelism": f"tp{world}",
        "allreduce": (args.allreduce if world > 1 else None),
        "fusions": (None if fuse_mode == "off" else
                    fuse_mode + ": RMSNorm->q/k/v, o+residual, RMSNorm->gate/up, SwiGLU->down+residual, "
                                "RMSNorm->head"),
        "attention": (None if fuse_mode == "off" or args.attention == "off" else
                      f"RoPE q,k; {args.attention} KV cache update; GQA attention over {args.context} "
                      f"positions ({cfg['heads']} heads / {cfg['kv_heads']} KV heads of {cfg['head_dim']})"),
        "weights_gb": round(job_bytes / 1e9, 3),
        "l2": "weights per step far above the 126 MB L2; no flush",
    }


def measure(args, torch, rank, world, local, dist):
    """One configuration: build this rank's stores, capture the step in a graph,
    time it, and return the JSON line (rank 0; None elsewhere)."""
    clq = importlib.import_module("cl-inference_b200")
    tp = importlib.import_module("cl-inference_b200.tp")
    cfg = dict(tp.LLAMA3_8B if args.model == "8b" else tp.LLAMA3_70B)
    if args.layers:
        cfg["layers"] = args.layers
    m = args.m
    xtype = args.xtype or ("f32" if m < 64 else "bf16")
    xdtype = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[xtype]
    prefill = m >= 64  # the tcgen05 GEMM: fp16 operands for 16-bit activations, the exact form for fp32
    exact = prefill and xtype == "f32"
    if args.workload != "step" and world > 1:
        raise SystemExit("GEMV sweeps run on one GPU")
    linears = workload_linears(args, tp, cfg)
    q_dim = cfg["heads"] * cfg["head_dim"]

    # ---- this rank's shards --------------------------------------------------
    stores, host_copies = [], []
    keep_host = world == 1 and not args.no_e2e
    for i, (name, dtype, n, k, kind, src) in enumerate(linears):
        s = tp.plan(dtype, n, k, kind, rank, world)
        if weights_kind(args) == "quantized":
            data = device_quantized_weight(torch, dtype, s.n, s.k, seed=4000 + 97 * i + rank)
        else:
            data = device_weight(torch, dtype, s.n, s.k, seed=4000 + 97 * i + rank)
        stores.append((clq.Store(dtype, s.n, s.k, data), s, dtype, kind, src, name))
        if keep_host:
            host_copies.append(data.cpu().numpy())
        del data
    torch.cuda.synchronize()

    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)
    attn_cols = tp.split(q_dim, world, rank, 256)
    ffn_cols = tp.split(cfg["ffn"], world, rank, 256)
    widths = {"hidden": cfg["hidden"], "attn": attn_cols[1] - attn_cols[0], "ffn": ffn_cols[1] - ffn_cols[0]}
    for (_, st, dt, kind, src, name) in stores:
        widths.setdefault(src, st.k)
    inputs = {src: torch.randn(m, w, device="cuda", generator=gen) for src, w in widths.items()}
    inputs = {key: v.to(xdtype) for key, v in inputs.items()}
    x_bytes = inputs[stores[0][4]].element_size()
    outs = [torch.empty(m, st.n, device="cuda") for (_, st, *_r) in stores]
    logits = torch.empty(world, m, stores[-1][1].n, device="cuda")
    # one launch per group of linears reading the same activations: per layer
    # (q, k, v), (o), (gate, up), (down); then the output head
    groups, i = [], 0
    if args.workload == "step":
        per_layer = len(tp.layer_linears(cfg))
        for layer in range(cfg["layers"]):
            base = layer * per_layer
            for members in ((0, 1, 2), (3,), (4, 5), (6,)):
                groups.append([base + j for j in members])
        groups.append([len(stores) - 1])
    else:
        groups = [[j] for j in range(len(stores))]
    launches_per_step = len(groups)

    def run_group(idx):
        if len(idx) == 1:
            store, s, dtype, kind, src, name = stores[idx[0]]
            store.linear(inputs[src], out=outs[idx[0]])
        else:
            src = stores[idx[0]][4]
            clq.linear_group([stores[j][0] for j in idx], inputs[src], outs=[outs[j] for j in idx])

    comm = None
    if dist is not None and args.allreduce == "fused":
        tpcomm = importlib.import_module("cl-inference_b200.tpcomm")

        def exchange(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got
        comm = tpcomm.TpComm(rank, world, exchange, cap=max(4096, 16 * m * (cfg["hidden"] // 16 // 100 + 1)))

    fuse_mode = args.fusions if (args.workload == "step" and world == 1) else "off"
    if fuse_mode != "off":
        if xdtype != torch.float32:
            raise SystemExit("--fusions runs the fp32 decode data flow")
        # the residual stream (each layer's input, updated in place), the RMSNorm
        # weights, and the layer data flow of local/blocks.lisp:115-116, 151-154,
        # 387-392; every step restarts from the same stream
        hidden = cfg["hidden"]
        resid0 = torch.randn(m, hidden, device="cuda", generator=gen)
        resid = resid0.clone()
        norm_w = torch.rand(hidden, device="cuda", generator=gen) + 0.5
        per_layer = len(tp.layer_linears(cfg))

        def rms(v):
            return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-5) * norm_w

        attn = args.attention if args.attention != "off" else None
        heads, kvh, hd = cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
        kv_dim = kvh * hd
        if attn:
            att = importlib.import_module("cl-inference_b200.attention")
            ctx = args.context
            if ctx < m:
                raise SystemExit("--context must hold the step's rows")
            pos0 = ctx - m  # the step's rows take the last positions; each step rewrites them
            cache = att.KVCache(ctx, cfg["layers"], kvh, hd, attn)
            for layer in range(cfg["layers"]):  # the prompt's keys and values, once
                if pos0:
                    kv = torch.randn(2, pos0, kvh, hd, device="cuda", generator=gen)
                    cache.update(layer, kv[0], kv[1], 0, check=True)
            qkv = torch.empty(m, q_dim + 2 * kv_dim, device="cuda")
            attn_out = torch.empty(m, q_dim, device="cuda")
            for layer in range(cfg["layers"]):
                b = layer * per_layer
                outs[b], outs[b + 1], outs[b + 2] = (qkv[:, :q_dim], qkv[:, q_dim:q_dim + kv_dim],
                                                     qkv[:, q_dim + kv_dim:])

        def attention(layer, b):
            """RoPE on q and k (one call over their adjacent heads), the cache
            update, attention over the context; the o projection's input."""
            if not attn:
                return inputs["attn"]
            att.rope(qkv[:, :q_dim + kv_dim].view(m, heads + kvh, hd), pos0, 500000.0)
            cache.update(layer, qkv[:, q_dim:q_dim + kv_dim].view(m, kvh, hd),
                         qkv[:, q_dim + kv_dim:].view(m, kvh, hd), pos0)
            att.attend(qkv[:, :q_dim].view(m, heads, hd), cache, layer, ctx, pos0, out=attn_out)
            return attn_out

        def step():
            resid.copy_(resid0)
            for layer in range(cfg["layers"]):
                b = layer * per_layer
                q, kk, v, o, gt, up, dn = (stores[b + j][0] for j in range(7))
                if fuse_mode == "fused":
                    clq.linear_group_fused([q, kk, v], resid, norm_weight=norm_w, eps=1e-5,
                                           outs=[outs[b], outs[b + 1], outs[b + 2]])
                    clq.linear_fused(o, attention(layer, b), out=resid, residual=resid)
                    clq.linear_group_fused([gt, up], resid, norm_weight=norm_w, eps=1e-5,
                                           outs=[outs[b + 4], outs[b + 5]])
                    clq.linear_fused(dn, outs[b + 5], gate=outs[b + 4], out=resid, residual=resid)
                else:
                    clq.linear_group([q, kk, v], rms(resid), outs=[outs[b], outs[b + 1], outs[b + 2]])
                    o.linear(attention(layer, b), out=outs[b + 3])
                    resid.add_(outs[b + 3])
                    clq.linear_group([gt, up], rms(resid), outs=[outs[b + 4], outs[b + 5]])
                    dn.linear(torch.nn.functional.silu(outs[b + 4]) * outs[b + 5], out=outs[b + 6])
                    resid.add_(outs[b + 6])
            head = stores[-1][0]
            if fuse_mode == "fused":
                clq.linear_fused(head, resid, norm_weight=norm_w, eps=1e-5, out=outs[-1])
            else:
                head.linear(rms(resid), out=outs[-1])
    else:
        def step():
            step_linears()

    nccl_fallback = set()  # row-parallel linears the fused all-reduce GEMV does not take

    def step_linears():
        for idx in groups:
            if comm is not None and stores[idx[0]][3] == "cols" and idx[0] not in nccl_fallback:
                store = stores[idx[0]][0]
                try:
                    comm.linear_allreduce(store, inputs[stores[idx[0]][4]], out=outs[idx[0]])
                    continue
                except clq.ClqError as exc:
                    # a shape the fused kernel does not plan (the same on every
                    # rank, so every rank takes the same collective path)
                    if exc.status != "CLQ_ERR_UNSUPPORTED":
                        raise
                    nccl_fallback.add(idx[0])
            run_group(idx)
            if dist is not None and stores[idx[0]][3] == "cols":
                dist.all_reduce(outs[idx[0]])
        if dist is not None:
            dist.all_gather_into_tensor(logits, outs[-1])

    # algorithmic bytes (W + x + out) of this rank's step, summed over ranks
    def lin_bytes(st, dtype):
        return tp.weight_bytes(dtype, st.n, st.k) + x_bytes * m * st.k + 4 * m * st.n
    step_bytes = float(sum(lin_bytes(st, dt) for (_, st, dt, *_r) in stores))
    if fuse_mode != "off" and args.attention != "off":
        # each layer reads the cached keys and values of the whole context
        per_row = cfg["head_dim"] * 4 if args.attention == "f32" else cfg["head_dim"] + 4 * -(-cfg["head_dim"] // 32)
        step_bytes += float(cfg["layers"] * 2 * args.context * cfg["kv_heads"] * per_row)
    if dist is not None:
        t = torch.tensor([step_bytes], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        job_bytes = float(t.item())
    else:
        job_bytes = step_bytes

    # ---- warm up eagerly (NCCL communicators), then capture a graph ----------
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph(keep_graph=True)
    with torch.cuda.graph(graph):
        step()
    try:
        ours_per_step, kernels_per_step = count_kernel_nodes(graph)
    except Exception as exc:  # launch count unavailable: say so rather than guess
        ours_per_step, kernels_per_step = None, None
        print(f"kernel-node count failed: {exc!r}", file=sys.stderr)
    graph.instantiate()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()

    # ---- timed region ---------------------------------------------------------
    clocks = ClockSampler(local)
    clocks.start()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clock = clocks.result()
    ms = start.elapsed_time(end) / args.steps
    if dist is not None:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    gbs = job_bytes / (ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    # the outputs of the last timed step, checked against float64 products
    check = None
    if fuse_mode == "off":
        check = check_outputs(torch, stores, outs, inputs, m, prefill and not exact, world, wide=prefill)
        if dist is not None:
            t = torch.tensor([check["max_rel_err"], 0.0 if check["element_bound_ok"] else 1.0],
                             dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            check["max_rel_err"] = float(t[0].item())
            check["element_bound_ok"] = bool(t[1].item() == 0.0)
            check["passed"] = check["element_bound_ok"] and check["max_rel_err"] <= 1e-3

    # ---- dominant kernel: the Q4_K GEMV launches alone, back to back ----------
    by_dtype = {}
    for (_, st, dt, *_r) in stores:
        by_dtype[dt] = by_dtype.get(dt, 0) + tp.weight_bytes(dt, st.n, st.k)
    top = "q4_k" if "q4_k" in by_dtype and args.workload == "step" else max(by_dtype, key=by_dtype.get)
    q4k_groups = [idx for idx in groups if stores[idx[0]][2] == top]
    kgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(kgraph):
        for idx in q4k_groups:
            run_group(idx)
    reps = max(5, min(50, args.steps // 5))
    for _ in range(3):
        kgraph.replay()
    torch.cuda.synchronize()
    ks, ke = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ks.record()
    for _ in range(reps):
        kgraph.replay()
    ke.record()
    torch.cuda.synchronize()
    k_ms = ks.elapsed_time(ke) / (reps * len(q4k_groups))
    k_bytes = sum(lin_bytes(stores[j][1], top) for idx in q4k_groups for j in idx) / len(q4k_groups)
    k_gbs = k_bytes / (k_ms * 1e-3) / 1e9
    k_flops = sum(2.0 * m * stores[j][1].n * stores[j][1].k for idx in q4k_groups for j in idx) / len(q4k_groups)
    step_flops = sum(2.0 * m * st.n * st.k for (_, st, *_r) in stores)
    traffic = None
    tfile = ROOT / "profiles" / "q4k_gemv_traffic.json"
    if tfile.exists() and world == 1 and m == 1 and args.model == "8b":  # the capture's shapes
        traffic = json.loads(tfile.read_text()).get("dram_bytes_per_launch_8b_step_avg")

    # ---- end to end -------------------------------------------------------------
    e2e = None
    if not args.no_e2e:
        e2e = e2e_dropin(args, clq, stores, host_copies, m, job_bytes, prefill and not exact) if world == 1 else \
            e2e_tp(args, torch, dist, graph, inputs, logits, job_bytes)

    del graph, kgraph
    if comm is not None:
        torch.cuda.synchronize()
        comm.close(barrier=dist.barrier)
    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": ("synthetic: N(0, 0.02) weights quantized to Q4_K / Q6_K on the device (synth.py), N(0,1) "
                     "activations" if weights_kind(args) == "quantized" else
                     "synthetic: uniform codes, |N(0,1)|-scaled fp16 scales, N(0,1) activations"),
            "config": config_dict(args, cfg, m, xtype, prefill, world, fuse_mode, job_bytes, len(stores)),
            "tok_per_s": round(1000.0 * m / ms, 2),
            "hbm_frac": round(gbs / world / peak, 4),
            "gpu_launches": ours_per_step * args.steps if ours_per_step is not None else None,
            "gpu_launches_per_step": {"clq": ours_per_step, "all_kernel_nodes": kernels_per_step},
            "clocks": clock,
            "check": check,
            "allreduce_nccl_fallbacks": len(nccl_fallback) if comm is not None else None,
            "libraries_mapped": repo_libraries(),
        }
        if prefill:
            tpeak, tpeak_kind = peak_tflops()
            k_tf = k_flops / (k_ms * 1e-3) / 1e12
            result["tflops"] = round(step_flops * world / (ms * 1e-3) / 1e12, 1)
            result["roofline"] = {
                "bound": "tensor", "kernel": ("Q4_K linears (activation prep + exact tcgen05 GEMM: three fp16 MMAs "
                                              "per K step + split-K reduce), " if exact else
                                              "Q4_K linears (activation prep + tcgen05 GEMM + split-K reduce), ")
                                             + "M=%d" % m,
                "achieved": round(k_tf, 1), "peak": tpeak, "peak_kind": tpeak_kind + " (burst, dense bf16)",
                "unit": "TFLOP/s", "frac": round(k_tf / tpeak, 4), "traffic": None,
                "algorithmic_flops_per_launch": round(k_flops), "us_per_launch": round(k_ms * 1e3, 3)}
        else:
            result["roofline"] = {
                "bound": "hbm", "kernel": ("Q4_K GEMV launches (q/k/v group, o, gate/up group), M=%d" % m)
                if args.workload == "step" else f"{top.upper()} GEMV launches of the sweep, M={m}",
                "achieved": round(k_gbs, 1), "peak": peak, "peak_kind": peak_kind,
                "unit": "GB/s", "frac": round(k_gbs / peak, 4), "traffic": traffic,
                "algorithmic_bytes_per_launch": round(k_bytes), "us_per_launch": round(k_ms * 1e3, 3)}
        if e2e:
            result["e2e"] = e2e
        if world == 1 and not args.no_cpu:
            result["cpu_baseline"] = cpu_baseline(args, tp, cfg, m)
    if dist is not None:
        dist.barrier()
    for entry in stores:
        entry[0].close()
    return result



def e2e_dropin(args, clq, stores, host_copies, m, job_bytes, prefill=False):
    """The host-buffer C ABI (clq_q4_k_matmul & co.), one synchronous call per linear.
    Prefill passes CLQ_MATH_FAST through clq_matmul so the fp32 host activations
    take the tensor-core GEMM."""
    import functools
    import numpy as np
    lib = clq._lib.lib
    if prefill:
        ggml = {"q4_0": 2, "q8_0": 8, "q4_k": 12, "q6_k": 14}
        fns = {d: functools.partial(lambda t, *a: lib.clq_matmul(t, *a, 1), g) for d, g in ggml.items()}
    else:
        fns = {"q4_k": lib.clq_q4_k_matmul, "q6_k": lib.clq_q6_k_matmul,
               "q8_0": lib.clq_q8_0_matmul, "q4_0": lib.clq_q4_0_matmul}
    rng = np.random.default_rng(3)
    xs = {}
    outs = []
    calls = []
    h2d = d2h = 0
    for (store, s, dtype, kind, src, name), data in zip(stores, host_copies):
        key = (src, s.k)
        if key not in xs:
            xs[key] = rng.standard_normal((m, s.k), dtype=np.float32)
        out = np.empty((m, s.n), np.float32)
        outs.append(out)
        # the buffers' addresses, as a foreign caller holds them (outs, xs and
        # host_copies keep the arrays alive)
        calls.append((fns[dtype], out.ctypes.data, xs[key].ctypes.data, data.ctypes.data, s.n, s.k))
        h2d += 4 * m * s.k
        d2h += 4 * m * s.n

    def one():
        for fn, out, x, data, n, k in calls:
            rc = fn(out, x, data, m, n, k)
            if rc:
                raise clq.ClqError(rc, clq._lib.last_error())

    for _ in range(3):
        one()  # first call uploads each weight once (cached by host range)
    steps = max(5, min(args.steps, 50))
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    sec = (time.perf_counter() - t0) / steps
    lib.clq_clear_cache()
    return {"value": round(job_bytes / sec / 1e9, 1), "unit": "GB/s", "ms_per_step": round(sec * 1e3, 4),
            "tok_per_s": round(1.0 / sec, 2), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": ("clq_matmul(CLQ_MATH_FAST)" if prefill else "clq_q4_k_matmul/clq_q6_k_matmul")
                   + ", host buffers, one synchronous call per linear",
            "steps": steps}


def e2e_tp(args, torch, dist, graph, inputs, logits, job_bytes):
    """Per step: pinned host input -> device, the captured tensor-parallel step, logits -> host."""
    host_in = torch.randn(inputs["hidden"].shape, pin_memory=True)
    host_out = torch.empty(logits.shape, pin_memory=True)
    steps = max(5, min(args.steps, 100))
    for _ in range(3):
        inputs["hidden"].copy_(host_in, non_blocking=True)
        graph.replay()
        host_out.copy_(logits, non_blocking=True)
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        inputs["hidden"].copy_(host_in, non_blocking=True)
        graph.replay()
        host_out.copy_(logits, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    sec = (time.perf_counter() - t0) / steps
    t = torch.tensor([sec], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    sec = float(t.item())
    return {"value": round(job_bytes / sec / 1e9, 1), "unit": "GB/s", "ms_per_step": round(sec * 1e3, 4),
            "tok_per_s": round(1.0 / sec, 2), "h2d_bytes_per_step": host_in.numel() * 4,
            "d2h_bytes_per_step": host_out.numel() * 4,
            "api": "tensor-parallel step (clq_linear_device + NCCL) with pinned host input/logits",
            "steps": steps}


def host_threads():
    """Every host core this process may run on (torchrun sets OMP_NUM_THREADS=1,
    so OpenMP's own default would undercount)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(tp, cfg, m, workload="step"):
    """Host bytes (numpy seeded) of a bounded sample of the workload: one decoder
    layer's seven linears for the decode step, one copy of each shape for a sweep."""
    synth = importlib.import_module("cl-inference_b200.synth")
    sample = []
    shapes = [(d, n, k) for (_, d, n, k, _, _) in tp.layer_linears(cfg)] if workload == "step" else SWEEPS[workload]
    for i, (dtype, n, k) in enumerate(shapes):
        data = synth.packed_blocks(dtype, n, k, seed=8000 + i)
        x = synth.activations(m, k, seed=8100 + i)
        sample.append((dtype, n, k, data, x))
    nbytes = sum(tp.weight_bytes(d, n, k) + 4 * m * k + 4 * m * n for d, n, k, _, _ in sample)
    return sample, nbytes


def time_cpu(sample, nbytes, seconds, threads):
    import oracle
    runs, t0 = 0, time.perf_counter()
    while True:
        for dtype, n, k, data, x in sample:
            oracle.matmul_f32(dtype, x, data, n, threads)
        runs += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            return runs * nbytes / el / 1e9, runs, el


def sample_name(workload):
    return "one layer's 7 linears" if workload == "step" else f"one copy of each {workload} shape"


def cpu_baseline(args, tp, cfg, m):
    sample, nbytes = cpu_sample(tp, cfg, m, args.workload)
    threads = host_threads()
    gbs, runs, el = time_cpu(sample, nbytes, args.cpu_seconds, threads)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{sample_name(args.workload)} ({nbytes/1e6:.1f} MB) x {runs} in {el:.1f} s, "
                      f"fp32 CPU port of the packed kernel contract, OpenMP"}


def workload_modules():
    """The package's shape tables (tp) and synthetic weights (synth) without
    running its __init__, which loads libclq.so: the reference arm maps no
    code of this library."""
    import types
    name = "cl-inference_b200"
    if name not in sys.modules:
        pkg = types.ModuleType(name)
        pkg.__path__ = [str(ROOT / name)]
        sys.modules[name] = pkg
    return importlib.import_module(name + ".tp"), importlib.import_module(name + ".synth")


def run_reference(args):
    """The reference arm: the CPU port of cl-inference's packed kernels
    (oracle/clq_oracle.c: the six-argument kernel contract of
    quant/packed.lisp:68-75 and quant/q8-0.lisp:77-85, fp32, OpenMP over every
    host core) on the same workload as the GPU arm -- every linear of the step,
    the same shapes and distributions -- timed per step.  Only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    tp, synth = workload_modules()
    import oracle
    cfg = dict(tp.LLAMA3_8B if args.model == "8b" else tp.LLAMA3_70B)
    if args.layers:
        cfg["layers"] = args.layers
    m = args.m
    linears = workload_linears(args, tp, cfg)
    widths = {}
    for (_, _, n, k, _, src) in linears:
        widths.setdefault(src, k)
    xs = {src: synth.activations(m, k, seed=8100 + i) for i, (src, k) in enumerate(sorted(widths.items()))}
    work = [(dtype, n, synth.packed_blocks(dtype, n, k, seed=8000 + i), xs[src])
            for i, (_, dtype, n, k, _, src) in enumerate(linears)]
    nbytes = float(sum(tp.weight_bytes(d, n, x.shape[1]) + 4 * m * x.shape[1] + 4 * m * n for d, n, _, x in work))
    threads = host_threads()

    def step():
        for dtype, n, data, x in work:
            oracle.matmul_f32(dtype, x, data, n, threads)

    warm0 = time.perf_counter()
    for _ in range(args.warmup):  # page-in and thread start-up
        step()
        if time.perf_counter() - warm0 > 60:
            break
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if sum(times) > 90:  # a bounded sample of the K steps asked for
            break
    sec = sum(times) / len(times)
    gbs = nbytes / sec / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": len(times), "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: uniform codes and random fp16 scales (the CPU kernel's time does not depend on the values)",
        "config": config_dict(args, cfg, m, "f32", False, 1, "off", nbytes, len(work)),
        "tok_per_s": round(m / sec, 4),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"the whole step ({nbytes / 1e9:.3f} GB of packed weights, {len(work)} linears) "
                                   f"per step, {len(times)} of the {args.steps} steps asked for (90 s cap)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "cl-inference's CPU kernels (trivial-simd, Common Lisp host) cannot be built here; "
                "this is the C port of their contract (oracle/clq_oracle.c) on the host cores",
        "libraries_mapped": repo_libraries(),
    }
    print(json.dumps(line), flush=True)


def repo_libraries():
    """This repository's shared libraries mapped into the process."""
    try:
        with open("/proc/self/maps") as f:
            paths = {ln.split()[-1] for ln in f if ln.rstrip().endswith(".so")}
    except OSError:
        return None
    return sorted(os.path.relpath(p, ROOT) for p in paths if p.startswith(str(ROOT) + os.sep))


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_clq(args)


if __name__ == "__main__":
    main()
