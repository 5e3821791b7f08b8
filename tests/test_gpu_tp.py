"""The fused GEMV + all-reduce over peer memory (needs a B200; two for the multi-rank case).

A group of one rank runs the whole protocol (epoch-tagged words into its own
buffer, wait, sum) and must reproduce the plain product bit for bit.  With two
GPUs, two processes each hold a K-slice of a row-parallel weight; every rank's
fused result must match the unsharded oracle product, over repeated calls that
exercise both buffer parities.
"""
import importlib
import os
import socket
import sys

import numpy as np
import pytest

from helpers import NORM_REL, max_row_relative_error

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_single_rank_group_reproduces_the_plain_product(cuda, clq, synth):
    torch = cuda
    tpcomm = importlib.import_module("cl-inference_b200.tpcomm")
    comm = tpcomm.TpComm(0, 1, lambda obj: [obj])
    try:
        for dtype, n, k in [("q4_k", 4096, 4096), ("q6_k", 1000, 2048)]:
            store = clq.Store(dtype, n, k, synth.packed_blocks(dtype, n, k, seed=n))
            for m in (1, 2, 5):
                for call in range(3):  # both buffer parities
                    x = torch.from_numpy(synth.activations(m, k, seed=10 * m + call)).cuda()
                    want = store.linear(x)
                    got = comm.linear_allreduce(store, x)
                    torch.cuda.synchronize()
                    assert torch.equal(got, want), (dtype, m, call)
            store.close()
        status = __import__("ctypes").c_int(-1)
        assert clq._lib.lib.clq_device_status(__import__("ctypes").byref(status)) == 0
        assert status.value == 0
    finally:
        comm.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    try:
        for p in (ROOT, os.path.join(ROOT, "oracle")):
            if p not in sys.path:
                sys.path.insert(0, p)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        clq = importlib.import_module("cl-inference_b200")
        tp = importlib.import_module("cl-inference_b200.tp")
        tpcomm = importlib.import_module("cl-inference_b200.tpcomm")
        synth = importlib.import_module("cl-inference_b200.synth")

        def exchange(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out
        comm = tpcomm.TpComm(rank, world, exchange)
        results = []
        for dtype, n, k in [("q4_k", 4096, 4096), ("q6_k", 2048, 4096)]:
            data = synth.packed_blocks(dtype, n, k, seed=n + k)
            s = tp.plan(dtype, n, k, "cols", rank, world)
            store = clq.Store(dtype, s.n, s.k, tp.shard_bytes(dtype, n, k, data, s))
            for call, m in enumerate((1, 3, 1, 8)):
                x = synth.activations(m, k, seed=100 * call + m)
                xs = torch.from_numpy(np.ascontiguousarray(x[:, s.col_begin:s.col_begin + s.k])).cuda()
                got = comm.linear_allreduce(store, xs)
                torch.cuda.synchronize()
                results.append((dtype, n, k, m, call, got.cpu().numpy()))
            store.close()
        comm.close(barrier=dist.barrier)
        dist.destroy_process_group()
        q.put((rank, results))
    except BaseException as exc:
        q.put((rank, repr(exc)))


def test_two_ranks_sum_their_shards_over_nvlink(cuda, clq, synth, oracle):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=300)
            got[r] = v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(got[r], str), got[r]
    for r in range(world):
        for dtype, n, k, m, call, out in got[r]:
            data = synth.packed_blocks(dtype, n, k, seed=n + k)
            x = synth.activations(m, k, seed=100 * call + m)
            ref, mag = oracle.matmul_f64(dtype, x, data, n)
            assert max_row_relative_error(out, ref) <= NORM_REL
            assert np.all(np.abs(out.astype(np.float64) - ref) <= 1e-5 + 1e-5 * mag)
    # both ranks hold the same sums
    for a, b in zip(got[0], got[1]):
        assert np.array_equal(a[-1], b[-1])
