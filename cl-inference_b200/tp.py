"""Tensor-parallel packed linears: row-sharded weights plus collectives.

cl-inference has no tensor parallelism (its only parallelism is the CPU
executor of docs/parallel-inference.md).  Here each rank of a process group
owns a slice of every packed weight, cut along whole GGUF blocks:

  column-parallel ("rows"): rank r owns weight rows [r*N/P, (r+1)*N/P); its
      output is the matching slice of out[m, N] (all-gathered when the caller
      needs the whole row, e.g. the logits);
  row-parallel ("cols"): rank r owns every row's blocks covering input columns
      [r*K/P, (r+1)*K/P); its output is a partial sum of out[m, N] that an
      all-reduce completes.

Megatron pairing uses column-parallel q/k/v/gate/up (their consumers, the
attention heads and the SwiGLU product, are sharded the same way) and
row-parallel o/down, so a decoder layer needs two all-reduces.  The slicing
here is host-side byte arithmetic on native blocks; the products are libclq
kernels and the collectives are torch.distributed (NCCL on GPUs).
"""
from dataclasses import dataclass

import numpy as np

from .geometry import find_dtype


@dataclass(frozen=True)
class Shard:
    kind: str        # "rows" (column-parallel) or "cols" (row-parallel)
    rank: int
    world: int
    n: int           # rows of this rank's packed matrix
    k: int           # columns of this rank's packed matrix
    row_begin: int   # first global output row (rows) / 0
    col_begin: int   # first global input column (cols) / 0


def split(total, world, rank, quantum=1):
    """[begin, end) of rank's share of TOTAL units, in multiples of QUANTUM."""
    if total % quantum:
        raise ValueError(f"{total} is not a multiple of {quantum}")
    units = total // quantum
    base, extra = divmod(units, world)
    begin = rank * base + min(rank, extra)
    end = begin + base + (1 if rank < extra else 0)
    return begin * quantum, end * quantum


def plan(dtype, n, k, kind, rank, world):
    dt = find_dtype(dtype)
    if kind == "rows":
        b, e = split(n, world, rank)
        return Shard("rows", rank, world, e - b, k, b, 0)
    if kind == "cols":
        b, e = split(k, world, rank, dt.block_size)
        return Shard("cols", rank, world, n, e - b, 0, b)
    raise ValueError(kind)


def shard_bytes(dtype, n, k, data, shard):
    """This rank's packed bytes (a valid N' x K' matrix) cut from the full weight."""
    dt = find_dtype(dtype)
    rows = np.asarray(data, np.uint8).reshape(n, k // dt.block_size * dt.block_bytes)
    if shard.kind == "rows":
        part = rows[shard.row_begin:shard.row_begin + shard.n]
    else:
        b0 = shard.col_begin // dt.block_size * dt.block_bytes
        b1 = (shard.col_begin + shard.k) // dt.block_size * dt.block_bytes
        part = rows[:, b0:b1]
    return np.ascontiguousarray(part).reshape(-1)


def assemble_rows(parts, shards, n):
    """Host-side gather of column-parallel outputs [m, n_r] into [m, n]."""
    m = parts[0].shape[0]
    out = np.empty((m, n), dtype=parts[0].dtype)
    for p, s in zip(parts, shards):
        out[:, s.row_begin:s.row_begin + s.n] = p
    return out


# ---- a decoder's packed linears, sharded (the benchmark workload) -----------

LLAMA3_8B = dict(hidden=4096, ffn=14336, heads=32, kv_heads=8, head_dim=128, layers=32, vocab=128256)
LLAMA3_70B = dict(hidden=8192, ffn=28672, heads=64, kv_heads=8, head_dim=128, layers=80, vocab=128256)


def layer_linears(cfg):
    """(name, dtype, n, k, tp kind, input buffer) of one Q4_K-M decoder layer.

    Q4_K_M recipe: Q4_K attention and gate/up, Q6_K down; the output head is Q6_K.
    """
    h, f = cfg["hidden"], cfg["ffn"]
    q, kv = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    return [
        ("attn_q", "q4_k", q, h, "rows", "hidden"),
        ("attn_k", "q4_k", kv, h, "rows", "hidden"),
        ("attn_v", "q4_k", kv, h, "rows", "hidden"),
        ("attn_output", "q4_k", h, q, "cols", "attn"),
        ("ffn_gate", "q4_k", f, h, "rows", "hidden"),
        ("ffn_up", "q4_k", f, h, "rows", "hidden"),
        ("ffn_down", "q6_k", h, f, "cols", "ffn"),
    ]


def model_linears(cfg):
    out = []
    for layer in range(cfg["layers"]):
        for name, dtype, n, k, kind, src in layer_linears(cfg):
            out.append((f"blk.{layer}.{name}", dtype, n, k, kind, src))
    out.append(("output", "q6_k", cfg["vocab"], cfg["hidden"], "rows", "hidden"))
    return out


def weight_bytes(dtype, n, k):
    dt = find_dtype(dtype)
    return n * (k // dt.block_size) * dt.block_bytes
