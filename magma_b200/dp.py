"""Data-parallel gradient synchronisation over torch.distributed (NCCL).

The reference averages per-replica gradients with ``crossReplicaMean``
(Sources/Core/Distributed.swift:55-64), lowered to ``all_reduce(add)`` followed
by a multiply by 1/n (MLIRBuilder.swift:923-929). Here the sum all-reduce runs
over the flat F32 gradient arena in fixed-size buckets, and the 1/n multiply is
folded into the Adam kernel's ``grad_scale`` (one pass over the gradients
fewer). One process per GPU; with world size 1 the sync is a no-op.
"""
from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def init_from_env(backend: str | None = None, timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Initialises the default process group from torchrun's environment.

    Returns (rank, world_size, local_rank). With WORLD_SIZE unset or 1 nothing
    is initialised.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, timeout=timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return rank, world, local


class GradSync:
    """Sum all-reduce of a flat gradient arena in buckets; returns 1/world.

    ``bucket_bytes`` bounds each collective (large buckets amortise launch
    latency; NVSwitch gives every peer full bandwidth, so link count does not
    enter the choice).
    """

    def __init__(self, group=None, bucket_bytes: int = 256 << 20):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.bucket_bytes = bucket_bytes

    def __call__(self, grads: torch.Tensor) -> float:
        if self.world == 1:
            return 1.0
        flat = grads.view(-1)
        per = max(1, self.bucket_bytes // flat.element_size())
        for start in range(0, flat.numel(), per):
            dist.all_reduce(flat[start:start + per], op=dist.ReduceOp.SUM, group=self.group)
        return 1.0 / self.world


def shard_batch(global_tokens: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [rank*b, (rank+1)*b) of a [world*b, S] batch (DistributedSampler's
    contiguous split, Data.swift:151-230)."""
    b = global_tokens.shape[0] // world
    return global_tokens[rank * b:(rank + 1) * b]
