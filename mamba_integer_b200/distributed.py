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


class LastLogitsGather:
    """All-gather of every rank's last-position logits [b_rank, V] into
    [global_batch, V] in global sequence order, with its buffers allocated once
    (per call: one copy into the send buffer, one all_gather_into_tensor, and
    for uneven shards one compaction copy per rank).

    Shards may be uneven (``shard_counts``): each rank sends a buffer padded to
    the largest shard, and the padding rows are dropped on the way out."""

    def __init__(self, global_batch: int, vocab: int, dtype=torch.float32, device=None):
        world = dist.get_world_size()
        self.rank = dist.get_rank()
        self.counts = shard_counts(global_batch, world)
        self.mx = max(self.counts)
        self.global_batch = global_batch
        self.send = torch.zeros(self.mx, vocab, dtype=dtype, device=device)
        self.recv = torch.empty(world * self.mx, vocab, dtype=dtype, device=device)
        self.even = all(c == self.mx for c in self.counts)
        self.out = self.recv if self.even else torch.empty(global_batch, vocab, dtype=dtype, device=device)

    def __call__(self, local_last: torch.Tensor) -> torch.Tensor:
        n = self.counts[self.rank]
        if local_last.shape[0] != n:
            raise ValueError(f"rank {self.rank} holds {local_last.shape[0]} rows, expected {n}")
        self.send[:n].copy_(local_last)
        dist.all_gather_into_tensor(self.recv, self.send)
        if self.even:
            return self.recv
        o = 0
        for r, c in enumerate(self.counts):
            self.out[o:o + c].copy_(self.recv[r * self.mx: r * self.mx + c])
            o += c
        return self.out


def gather_last_logits(local_last: torch.Tensor, global_batch: int) -> torch.Tensor:
    """All-gather every rank's last-position logits [b_rank, V] into [global_batch, V]
    in global sequence order (handles uneven shards by padding to the largest)."""
    g = LastLogitsGather(global_batch, local_last.shape[1], local_last.dtype, local_last.device)
    return g(local_last).clone()


def gather_ids(local_ids: torch.Tensor, global_batch: int) -> torch.Tensor:
    """All-gather every rank's generated token ids [b_rank, steps] (int64) into
    [global_batch, steps] in global stream order (uneven shards padded)."""
    world = dist.get_world_size()
    counts = shard_counts(global_batch, world)
    mx = max(counts)
    steps = local_ids.shape[1]
    buf = torch.zeros(mx, steps, dtype=local_ids.dtype, device=local_ids.device)
    buf[: local_ids.shape[0]] = local_ids
    out = torch.empty(world * mx, steps, dtype=local_ids.dtype, device=local_ids.device)
    dist.all_gather_into_tensor(out, buf)
    return torch.cat([out[r * mx: r * mx + counts[r]] for r in range(world)], 0)
