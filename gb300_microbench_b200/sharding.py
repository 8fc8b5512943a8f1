"""Row sharding of the GEMM across GPUs (one process per GPU).

Rank r of P owns rows [row0, row0 + rows) of A and C; B is replicated. Each
rank runs the single-GPU kernel on its (rows, N, K) block, so the timed
path has no collective. ``gather_rows`` reassembles C on every rank with one
all-gather for validation only (NCCL on GPUs, gloo in the CPU tests).

This is the multi-GPU mode this build adds to the reference,
which is strictly single-GPU (memory_paths/ldgsts.cu:396-398,
gemm_comparison.py:1098-1108).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch


@dataclass(frozen=True)
class RowShard:
    rank: int
    world: int
    row0: int
    rows: int


def row_shard(m: int, world: int, rank: int, granule: int = 1) -> RowShard:
    """Contiguous, balanced row blocks; block sizes are multiples of
    `granule` except possibly the last. With fewer granules than ranks the
    lowest ranks hold them and the rest get empty blocks, so rank 0 always
    holds rows when m > 0."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world} is invalid")
    if m < 0 or granule < 1:
        raise ValueError("m must be >= 0 and granule >= 1")
    units = -(-m // granule)
    if units < world:
        u0, u1 = min(rank, units), min(rank + 1, units)  # one granule each to the lowest ranks
    else:
        u0 = rank * units // world
        u1 = (rank + 1) * units // world
    row0 = min(u0 * granule, m)
    row1 = min(u1 * granule, m)
    return RowShard(rank, world, row0, row1 - row0)


def gather_rows(local: torch.Tensor, shards: list[RowShard], group=None) -> torch.Tensor:
    """All-gathers the per-rank row blocks of C into the full matrix
    (validation only; never inside a timed region)."""
    import torch.distributed as dist

    world = len(shards)
    cols = local.shape[1]
    max_rows = max(s.rows for s in shards)
    padded = torch.zeros(max_rows, cols, dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    bufs = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(bufs, padded, group=group)
    return torch.cat([bufs[s.rank][: s.rows] for s in shards], dim=0)


def sharded_gemm(a_full: torch.Tensor, b: torch.Tensor, world: int, rank: int,
                 gemm_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor], granule: int = 128,
                 gather: bool = True):
    """Runs C = A B^T with A row-sharded over `world` ranks. `gemm_fn(a_block,
    b)` computes one block (the native GEMM on a GPU). Returns (local C block,
    full C or None, the shard)."""
    shards = [row_shard(a_full.shape[0], world, r, granule) for r in range(world)]
    me = shards[rank]
    c_local = gemm_fn(a_full[me.row0: me.row0 + me.rows], b)
    full = gather_rows(c_local, shards) if gather and world > 1 else (c_local if world == 1 else None)
    return c_local, full, me
