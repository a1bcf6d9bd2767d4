"""Sequence sharding across GPUs and rank-level reductions for multi-GPU runs.

Each GPU holds a full model replica and decodes its own sequences; the data path
has no collective (independent sequences: "replicas only").
The only cross-rank traffic is host bookkeeping: which sequences a rank owns and
the max over ranks of a device-timed interval.  Works with any torch.distributed
backend (gloo on CPU, nccl on GPUs).
"""
from __future__ import annotations


def shard_sequences(num_seqs: int, world: int, rank: int) -> list[int]:
    """Round-robin partition of sequence ids 0..num_seqs-1: rank r owns r, r+world, ..."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if num_seqs < 0:
        raise ValueError("num_seqs must be >= 0")
    return list(range(rank, num_seqs, world))


def max_over_ranks(value: float, device: str = "cpu") -> float:
    """Max of a per-rank float over the default process group (identity without one)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device: str = "cpu") -> float:
    """Sum of a per-rank float over the default process group (identity without one)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
