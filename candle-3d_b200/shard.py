"""Row sharding across ranks (one process per GPU).

Every per-token op is independent per row, so rank r of W owns the contiguous
row range `shard_range(n, W, r)` and runs the fused kernels on it with no
communication.  `gather_rows` is the optional final all-gather of the block
outputs (uneven shards are padded to the largest shard for the collective and
trimmed afterwards); it works with any torch.distributed backend (NCCL on the
GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's rows; the first n % world ranks get one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def gather_rows(local: torch.Tensor, n: int, world: int, group=None) -> torch.Tensor:
    """All-gather row shards [rows_r, ...] into the full [n, ...] tensor on every rank."""
    if world == 1:
        return local
    cap = shard_range(n, world, 0)[1]  # the largest shard
    padded = local.new_zeros((cap,) + tuple(local.shape[1:]))
    padded[: local.shape[0]] = local
    out = local.new_empty((world * cap,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(out, padded, group=group)
    parts = [out[r * cap: r * cap + (shard_range(n, world, r)[1] - shard_range(n, world, r)[0])]
             for r in range(world)]
    return torch.cat(parts, 0)
