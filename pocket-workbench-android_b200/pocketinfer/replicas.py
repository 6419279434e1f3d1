"""Host-side plumbing for N independent decode replicas (one process per GPU).

b = 1 decode of one stream does not shard, so N GPUs run N replicas with no
data-path collective.  The only cross-rank step is timing: every rank times
its own steps on its device, and the job's throughput uses the slowest rank.
"""
from __future__ import annotations


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Maximum of a per-rank float over the default process group (or the value itself)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def replica_throughput(steps_per_rank: int, local_ms: float, world: int, dist=None, device=None):
    """(aggregate units/s, max-over-ranks ms) for `world` replicas of `steps_per_rank` units each."""
    ms = max_over_ranks(local_ms, dist, device)
    if ms <= 0.0:
        raise ValueError("non-positive timed region")
    return world * steps_per_rank / (ms / 1000.0), ms


def assign_streams(n_streams: int, rank: int, world: int) -> list:
    """Independent request streams of a data-parallel run, dealt round-robin to ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    return list(range(rank, n_streams, world))
