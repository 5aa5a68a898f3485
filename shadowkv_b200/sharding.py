"""Sharding of the decode step across the GPUs of one node.

Every (sequence, kv head) unit of the step is independent -- scoring,
selection, reuse cache, reconstruction and attention never mix units -- so
the step shards two ways without any exchange inside the path:

* by sequence: rank r owns sequences ``batch_range(B, world, r)`` with all
  their heads (its own pinned value store, its own GPU); nothing is
  exchanged;
* by kv head: rank r owns kv heads ``head_range(Hkv, world, r)`` and the
  query heads of their GQA groups; the attention outputs of the head shards
  are all-gathered (NCCL over NVLink) before the output projection, which
  needs every head (``gather_head_shards``).

Timing helpers take the max over ranks, as a multi-GPU step is as slow as
its slowest rank.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def batch_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """(first sequence, count) of ``rank``; the counts differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, rem = divmod(batch, world)
    count = base + (1 if rank < rem else 0)
    start = rank * base + min(rank, rem)
    return start, count


def head_range(kv_heads: int, q_heads: int, world: int, rank: int) -> tuple[int, int, int, int]:
    """(first kv head, kv count, first q head, q count) of ``rank``.

    kv heads must divide evenly: a GQA group never spans two ranks.
    """
    if kv_heads % world != 0:
        raise ValueError(f"{kv_heads} kv heads do not split over {world} ranks")
    g = q_heads // kv_heads
    per = kv_heads // world
    return rank * per, per, rank * per * g, per * g


def gather_head_shards(out_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather head shards ``[B, Hq/world, D]`` -> ``[B, Hq, D]`` (rank order = head order)."""
    world = dist.get_world_size(group)
    if world == 1:
        return out_local
    parts = [torch.empty_like(out_local) for _ in range(world)]
    dist.all_gather(parts, out_local.contiguous(), group=group)
    return torch.cat(parts, dim=1)


def max_over_ranks(value: float, device=None, group=None) -> float:
    """Max of a host scalar over the ranks of ``group`` (1 rank: identity)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
