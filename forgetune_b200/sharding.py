"""Batch sharding across ranks (one process per GPU).

Every forward row is independent, so a global batch splits into contiguous
row blocks with no exchange on the data path; the only cross-rank traffic is
the barrier around a timed region and the max-over-ranks of its duration.
The helpers work on any torch.distributed backend (NCCL on GPUs, gloo on CPU).
"""

from __future__ import annotations

import os
from datetime import timedelta
from typing import Optional, Tuple

import torch
import torch.distributed as dist


def rank_info() -> Tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment, (0, 1, 0) without it."""
    def env(name, default):
        try:
            return int(os.environ.get(name, default))
        except ValueError:
            return default
    return env("RANK", 0), env("WORLD_SIZE", 1), env("LOCAL_RANK", 0)


def shard_rows(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous row block [r0, r1) of `rank`: ceil(batch / world) rows each, the tail on the last ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank %d outside world of %d" % (rank, world))
    per = (batch + world - 1) // world
    r0 = min(batch, rank * per)
    return r0, min(batch, r0 + per)


def shard_element_offset(rank: int, rows_per_rank: int, features: int) -> int:
    """First global element index of a rank's input shard (weak scaling: equal shards)."""
    return rank * rows_per_rank * features


def init(backend: str, device: Optional[torch.device] = None, timeout_s: float = 300.0) -> None:
    """Initialise the default process group (short timeout so a lost rank ends collectives with an error)."""
    kw = {"backend": backend, "timeout": timedelta(seconds=timeout_s)}
    if device is not None and device.type == "cuda":
        kw["device_id"] = device
    dist.init_process_group(**kw)


def barrier() -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def max_over_ranks(value: float, device: Optional[torch.device] = None) -> float:
    """Maximum of a per-rank float over all ranks (the slowest rank's time)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or torch.device("cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
