"""Replica sharding across ranks (one process per GPU).

The encoder forward has no cross-row interaction, so multi-GPU runs are
replicas: batches are dealt round-robin to ranks (batch i -> rank i % world)
and no collective touches the data path.  The only collectives are a
barrier and the max-reduction of each rank's device time.
"""
from __future__ import annotations


def init_replica_group(backend: str, timeout_s: float = 180.0, device_id=None) -> None:
    """The job's one process group, with a short timeout: a rank that died or
    never joined ends the others' next collective (or the rendezvous) with an
    error instead of a hang.  The replicas exchange nothing but a barrier and
    a max of timings, so no legitimate wait comes near the limit."""
    from datetime import timedelta

    import torch.distributed as dist
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if device_id is not None:
        kw["device_id"] = device_id
    dist.init_process_group(backend, **kw)


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
