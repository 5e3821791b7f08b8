"""Tensor-parallel sharding of packed weights (CPU, world size 2 over gloo).

Each rank cuts its shard out of the full packed weight (tp.plan / tp.shard_bytes),
computes its part with the oracle, and the ranks combine the parts with the
collective the benchmark uses: all-gather of column-parallel outputs (rows
kind), all-reduce of row-parallel partial sums (cols kind).  The combined
result must equal the unsharded oracle product.
"""
import importlib
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_split_partitions_exactly():
    tp = importlib.import_module("cl-inference_b200.tp")
    for total, quantum in [(4096, 1), (1024, 1), (14336, 256), (28672, 256), (128256, 1), (37, 1), (512, 32)]:
        for world in (1, 2, 3, 4, 8):
            ranges = [tp.split(total, world, r, quantum) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            for (b0, e0), (b1, _) in zip(ranges, ranges[1:]):
                assert e0 == b1
            sizes = [e - b for b, e in ranges]
            assert all(s % quantum == 0 for s in sizes)
            assert max(sizes) - min(sizes) <= quantum
    with pytest.raises(ValueError):
        tp.split(100, 2, 0, 32)


@pytest.mark.parametrize("cfg_name", ["LLAMA3_8B", "LLAMA3_70B"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_model_shards_cover_every_linear(cfg_name, world):
    tp = importlib.import_module("cl-inference_b200.tp")
    cfg = getattr(tp, cfg_name)
    for name, dtype, n, k, kind, src in tp.model_linears(dict(cfg, layers=1)):
        shards = [tp.plan(dtype, n, k, kind, r, world) for r in range(world)]
        if kind == "rows":
            assert sum(s.n for s in shards) == n and all(s.k == k for s in shards)
        else:
            assert sum(s.k for s in shards) == k and all(s.n == n for s in shards)
            assert all(s.k % 256 == 0 for s in shards)  # whole K-quant superblocks
        total = sum(tp.weight_bytes(dtype, s.n, s.k) for s in shards)
        assert total == tp.weight_bytes(dtype, n, k)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, case, q):
    """One gloo rank: shard, compute with the oracle, combine, send back."""
    try:
        for p in (ROOT, os.path.join(ROOT, "oracle")):
            if p not in sys.path:
                sys.path.insert(0, p)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist
        import oracle
        tp = importlib.import_module("cl-inference_b200.tp")
        synth = importlib.import_module("cl-inference_b200.synth")
        dist.init_process_group("gloo", rank=rank, world_size=world)
        dtype, n, k, m, kind = case
        data = synth.packed_blocks(dtype, n, k, seed=n + k)
        x = synth.activations(m, k, seed=m)
        s = tp.plan(dtype, n, k, kind, rank, world)
        part_bytes = tp.shard_bytes(dtype, n, k, data, s)
        xs = x[:, s.col_begin:s.col_begin + s.k] if kind == "cols" else x
        part, _ = oracle.matmul_f64(dtype, np.ascontiguousarray(xs), part_bytes, s.n)
        if kind == "rows":
            sizes = [tp.plan(dtype, n, k, kind, r, world).n for r in range(world)]
            bufs = [torch.zeros(m, sz, dtype=torch.float64) for sz in sizes]
            dist.all_gather(bufs, torch.from_numpy(part))
            full = torch.cat(bufs, dim=1).numpy()
        else:
            t = torch.from_numpy(part)
            dist.all_reduce(t)
            full = t.numpy()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, full))
    except BaseException as exc:  # report instead of hanging the parent
        q.put((rank, repr(exc)))


@pytest.mark.parametrize("case", [
    ("q4_k", 300, 1024, 3, "rows"),   # column-parallel, ragged rows per rank
    ("q6_k", 96, 1024, 2, "cols"),    # row-parallel, whole superblocks per rank
    ("q8_0", 64, 256, 1, "cols"),
])
def test_sharded_products_match_unsharded_over_gloo(oracle, synth, case):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, val = q.get(timeout=180)
            results[rank] = val
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(results[r], str), results[r]
    dtype, n, k, m, kind = case
    data = synth.packed_blocks(dtype, n, k, seed=n + k)
    x = synth.activations(m, k, seed=m)
    ref, mag = oracle.matmul_f64(dtype, x, data, n)
    for r in range(world):
        assert results[r].shape == (m, n)
        # row-parallel sums re-associate fp64 partial sums: relative 1e-12
        assert np.all(np.abs(results[r] - ref) <= 1e-12 * (mag + 1.0))
