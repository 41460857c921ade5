"""Replica sharding across ranks (one process per GPU).

The encoder forward has no cross-row interaction, so multi-GPU runs are
replicas: batches are dealt round-robin to ranks (batch i -> rank i % world)
and no collective touches the data path.  The only collectives are a
barrier and the max-reduction of each rank's device time.
"""
from __future__ import annotations


def shard_batches(n_batches: int, rank: int, world: int) -> list[int]:
    """Round-robin: the batch indices rank `rank` of `world` processes."""
    if not (0 <= rank < world):
        raise ValueError("rank out of range")
    return list(range(rank, n_batches, world))


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank float over the default process group (identity
    when torch.distributed is not initialised)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(units_per_rank: list[int] | int, world: int, seconds: float) -> float:
    """Units all ranks processed / the max-over-ranks time."""
    total = sum(units_per_rank) if isinstance(units_per_rank, list) else units_per_rank * world
    return total / seconds
