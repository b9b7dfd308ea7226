"""Batch partitioning across the GPUs of one node and the one collective of
the prefill path (the reference has no distributed code; sequences are
independent, so each rank runs a contiguous slice of the batch on a full
weight replica and only the last-position logits are exchanged).

One process per GPU (torchrun); NCCL over NVLink for the gather on GPUs, gloo
for the CPU tests of the same logic.
"""
from __future__ import annotations

import datetime
import os
from typing import List, Tuple

import torch
import torch.distributed as dist


def shard_counts(global_batch: int, world: int) -> List[int]:
    """Sequences per rank: as even as possible, the first ranks take the remainder."""
    if world <= 0 or global_batch < 0:
        raise ValueError("world must be positive and global_batch non-negative")
    base, rem = divmod(global_batch, world)
    return [base + (1 if r < rem else 0) for r in range(world)]


def shard_range(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """[lo, hi) of the sequences owned by ``rank``."""
    counts = shard_counts(global_batch, world)
    lo = sum(counts[:rank])
    return lo, lo + counts[rank]


def init_from_env(backend: str = "nccl", timeout_s: float = 120.0):
    """init_process_group from torchrun's environment with a short timeout so a
    missing or dead rank ends the collective with an error instead of a hang."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return world, rank


def gather_last_logits(local_last: torch.Tensor, global_batch: int) -> torch.Tensor:
    """All-gather every rank's last-position logits [b_rank, V] into [global_batch, V]
    in global sequence order (handles uneven shards by padding to the largest)."""
    world = dist.get_world_size()
    counts = shard_counts(global_batch, world)
    if local_last.shape[0] != counts[dist.get_rank()]:
        raise ValueError(f"rank {dist.get_rank()} holds {local_last.shape[0]} rows, expected {counts[dist.get_rank()]}")
    mx = max(counts)
    V = local_last.shape[1]
    buf = torch.zeros(mx, V, dtype=local_last.dtype, device=local_last.device)
    buf[: local_last.shape[0]] = local_last
    out = torch.empty(world * mx, V, dtype=local_last.dtype, device=local_last.device)
    dist.all_gather_into_tensor(out, buf)
    parts = [out[r * mx: r * mx + counts[r]] for r in range(world)]
    return torch.cat(parts, 0)
