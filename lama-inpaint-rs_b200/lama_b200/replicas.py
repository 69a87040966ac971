"""Replica data parallelism: one process per GPU, images dealt round-robin.

The big-lama pass does not shard (the FourierUnit's FFT is global over the
latent plane), so N GPUs run N independent replicas with their own weights and
no collectives on the data path.  The only cross-rank
operations are a barrier and the max-over-ranks reduction of the timed region.
"""

from __future__ import annotations


def shard(total: int, rank: int, world: int) -> list[int]:
    """Round-robin: image i belongs to rank i % world."""
    if not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world {world}")
    return list(range(rank, total, world))


def chunks(n: int, chunk: int) -> list[tuple[int, int]]:
    """(start, count) pieces of at most `chunk` images covering range(n)."""
    if chunk < 1:
        raise ValueError("chunk must be >= 1")
    return [(s, min(chunk, n - s)) for s in range(0, n, chunk)]


def max_over_ranks(value: float, world: int, device=None) -> float:
    """The slowest rank's time (the whole-job time of a replica run)."""
    if world <= 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
