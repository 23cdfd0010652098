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
        self._stream = None
        self._works = []

    def _buckets(self, grads: torch.Tensor):
        flat = grads.view(-1)
        per = max(1, self.bucket_bytes // flat.element_size())
        for start in range(0, flat.numel(), per):
            yield flat[start:start + per]

    def __call__(self, grads: torch.Tensor) -> float:
        if self.world == 1:
            return 1.0
        for b in self._buckets(grads):
            dist.all_reduce(b, op=dist.ReduceOp.SUM, group=self.group)
        return 1.0 / self.world

    def launch(self, grads: torch.Tensor) -> None:
        """Starts the sum all-reduce of one finished gradient range. On CUDA it
        runs on a communication stream that first waits for the work queued so
        far on the current stream, so the next backward segment overlaps it;
        finish() joins. Every rank must launch the same ranges in the same
        order. (CPU tensors: done synchronously.)"""
        if self.world == 1:
            return
        if not grads.is_cuda:
            for b in self._buckets(grads):
                dist.all_reduce(b, op=dist.ReduceOp.SUM, group=self.group)
            return
        if self._stream is None:
            self._stream = torch.cuda.Stream(grads.device)
        self._stream.wait_stream(torch.cuda.current_stream(grads.device))
        with torch.cuda.stream(self._stream):
            for b in self._buckets(grads):
                self._works.append(
                    dist.all_reduce(b, op=dist.ReduceOp.SUM, group=self.group, async_op=True))

    def finish(self) -> float:
        """Makes the current stream wait for every launched all-reduce and
        returns the 1/world scale for Adam."""
        if self.world == 1:
            return 1.0
        for w in self._works:
            w.wait()
        self._works = []
        if self._stream is not None:
            torch.cuda.current_stream(self._stream.device).wait_stream(self._stream)
        return 1.0 / self.world


def shard_batch(global_tokens: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [rank*b, (rank+1)*b) of a [world*b, S] batch (DistributedSampler's
    contiguous split, Data.swift:151-230)."""
    b = global_tokens.shape[0] // world
    return global_tokens[rank * b:(rank + 1) * b]
