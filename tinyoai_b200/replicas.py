"""Replica bookkeeping for data-parallel decode: one process per GPU.

Each rank holds its own copy of the weights and serves its own sequences.
The configs that shard (independent sessions, branches of a shared prefix)
partition whole sequences, so nothing crosses ranks on the step path. Only
timing is exchanged: the whole-job time is the slowest rank's, and
throughput is the work of all ranks over that time (weak scaling when each
rank's share is fixed).
"""
import os

import torch
import torch.distributed as dist


def world():
    """(world_size, rank, local_rank) from the torchrun environment."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def _active():
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def barrier():
    if _active():
        dist.barrier()


def max_over_ranks(values, device=None):
    """Element-wise maximum of a list of floats over all ranks (float64)."""
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if _active():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def aggregate_rate(units_per_rank, world_size, seconds):
    """Whole-job throughput: every rank's units over the slowest rank's time."""
    if seconds <= 0:
        raise ValueError("elapsed time must be positive")
    return world_size * units_per_rank / seconds


def shard(n, world_size, rank):
    """Contiguous share [lo, hi) of n independent items for one rank; the
    shares cover [0, n) exactly and differ in size by at most one."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("rank outside the world")
    return n * rank // world_size, n * (rank + 1) // world_size
