"""Batch sharding of independent rollouts across GPUs (one process per GPU).

The hot path has no exchange step: every rollout is independent, so B_total
observations are split into contiguous shards, each process runs its shard on
its own GPU with a full weight replica, and only the decoded chunks travel
back to the host.  This mirrors the reference's one-evaluator-worker-per-GPU
layout (eval/README.md:20-27) and the per-row seeding of its batched twin
(eval/native/fastwam_batched_infer.py:59-66).  torch.distributed carries only
the host-side gather of results and the max-over-ranks timing, never the data
path of a chunk.
"""
from __future__ import annotations

from typing import Callable, List, Sequence, Tuple

import torch


def shard_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of `total` rollouts owned by `rank` of `world`;
    the first total % world ranks take one extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def seeded_noise(seeds: Sequence[int], shape: Sequence[int], dtype=torch.float32) -> torch.Tensor:
    """One CPU generator per rollout (fastwam_batched_infer.py:59-66 draws per-row noise the
    same way), stacked to [len(seeds), *shape]."""
    out = []
    for s in seeds:
        g = torch.Generator(device="cpu").manual_seed(int(s))
        out.append(torch.randn(tuple(shape), generator=g, dtype=torch.float32).to(dtype))
    return torch.stack(out) if out else torch.empty((0, *shape), dtype=dtype)


def run_shard(fn: Callable[[int, int], torch.Tensor], total: int, world: int, rank: int,
              gather: bool = True, group=None) -> List[torch.Tensor]:
    """Run fn(start, stop) on this rank's shard; with gather=True rank 0 receives every
    shard's result (host tensors, in rank order) through torch.distributed."""
    start, stop = shard_range(total, world, rank)
    local = fn(start, stop).cpu() if stop > start else torch.empty(0)
    if world == 1 or not gather:
        return [local]
    import torch.distributed as dist
    parts: List = [None] * world
    dist.all_gather_object(parts, local, group=group)
    return parts


def max_over_ranks(value: float, device=None, group=None) -> float:
    """Max of a per-rank scalar (timings are reported as the slowest rank)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
