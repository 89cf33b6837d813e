"""Data parallelism over independent sequences (one process per GPU, torch.distributed for the plumbing only).

The hot path has no exchange step: every rank holds the whole model and decodes its own sequences.  The ranks meet
only to agree on the timing (the slowest rank's time is the job's) and to split a pool of sequences."""
from __future__ import annotations


def shard(n_total: int, rank: int, world: int) -> range:
    """The contiguous slice of n_total sequence ids rank owns (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def rank_seed(seed: int, rank: int) -> int:
    """Each rank's sequences are seeded apart (the same rank always gets the same prompts)."""
    return seed + 7919 * rank


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """The job's time: the maximum over ranks (a plain value without a process group)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
