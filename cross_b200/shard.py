"""Batch sharding across ranks (one process per GPU).

The reference's only parallelism is a batch NamedSharding over a device mesh
(util.py:40-58 create_sharding, profiler.py:319-326): ciphertexts are
independent, so every operator on the path is batch-local and ranks exchange
nothing on the data path.  This module holds the host side of that: the rank
environment, which ciphertexts a rank owns, the max-over-ranks timing
reduction, and an apply-and-gather helper for callers that hold a global batch.
Collectives go through torch.distributed (NCCL on GPUs, gloo on CPU).
"""
from __future__ import annotations

import os
from typing import Callable, Tuple


def rank_env() -> Tuple[int, int, int]:
    """(world_size, rank, local_rank) from the torchrun environment."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard_bounds(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, balanced [start, stop) of a batch of `total` ciphertexts for
    `rank` of `world` (the first total % world ranks take one extra)."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request total={total} world={world} rank={rank}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of `value` over all ranks (timing: the slowest rank sets the
    job time).  Without an initialised process group, `value` itself."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def apply_sharded(fn: Callable, batch, world: int, rank: int):
    """Runs fn on this rank's shard of `batch` (a tensor whose first axis is
    the ciphertext batch) and returns the full result, assembled on every rank
    in batch order with an all-gather.  fn must map a shard of b ciphertexts to
    a tensor whose first axis is b (its other axes equal on every rank)."""
    import torch
    import torch.distributed as dist
    start, stop = shard_bounds(batch.shape[0], world, rank)
    part = fn(batch[start:stop])
    if world == 1:
        return part
    sizes = [shard_bounds(batch.shape[0], world, r) for r in range(world)]
    width = max(b - a for a, b in sizes)
    padded = torch.zeros((width, *part.shape[1:]), dtype=part.dtype, device=part.device)
    padded[: part.shape[0]] = part
    gathered = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(gathered, padded)
    return torch.cat([g[: b - a] for g, (a, b) in zip(gathered, sizes)], dim=0)
