"""Data-parallel gradient synchronisation.

The reference averages per-replica gradients with ``crossReplicaMean``
(Sources/Core/Distributed.swift:55-64), lowered to ``all_reduce(add)`` followed
by a multiply by 1/n (MLIRBuilder.swift:923-929). Here the sum all-reduce runs
over the flat F32 gradient arena in fixed-size buckets, and the 1/n multiply is
folded into the Adam kernel's ``grad_scale`` (one pass over the gradients
fewer). One process per GPU; with world size 1 the sync is a no-op.

On the GPU the exchange goes through the library's own C-ABI collectives
(``magma_allreduce`` and friends over NCCL, with ``magma_event_*`` ordering the
communication stream after the compute stream): ``Comm`` is one rank's
communicator, created from an id that rank 0 makes and the process group
broadcasts. ``torch.distributed`` is used only to start the processes and to
hand that id around (and, for CPU tensors in the host-logic tests, as the gloo
transport).
"""
from __future__ import annotations

import ctypes as C
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from . import lib


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


_DT = {torch.float32: lib.F32, torch.bfloat16: lib.BF16, torch.int32: lib.S32,
       torch.int64: lib.S64}


class Comm:
    """This rank's communicator of libmagma_cuda.so (NCCL under the C ABI)."""

    def __init__(self, handle: C.c_void_p, rank: int, world: int):
        self.handle, self.rank, self.world = handle, rank, world

    @classmethod
    def from_process_group(cls, group=None, timeout_ms: int = 120_000) -> "Comm":
        """Rank 0 makes the id, the process group broadcasts it, every rank
        joins on its current CUDA device (bounded by timeout_ms)."""
        rank = dist.get_rank(group)
        world = dist.get_world_size(group)
        uid = C.create_string_buffer(lib.COMM_ID_BYTES)
        if rank == 0:
            lib.call("magma_comm_unique_id", uid, lib.COMM_ID_BYTES)
        box = [uid.raw if rank == 0 else None]
        dist.broadcast_object_list(box, src=0, group=group)
        uid = C.create_string_buffer(box[0], lib.COMM_ID_BYTES)
        h = C.c_void_p()
        lib.call("magma_comm_init_rank", C.byref(h), world, rank, uid, timeout_ms)
        return cls(h, rank, world)

    def check(self) -> None:
        """Raises MagmaError once the communicator has failed (e.g. a peer died)."""
        lib.call("magma_comm_check", self.handle)

    def allreduce(self, t: torch.Tensor, op: int = lib.REDUCE_SUM, out: torch.Tensor | None = None,
                  stream: int | None = None) -> torch.Tensor:
        out = t if out is None else out
        lib.call("magma_allreduce", t.data_ptr(), out.data_ptr(), t.numel(), _DT[t.dtype], op,
                 self.handle, _stream(t) if stream is None else stream)
        return out

    def reduce_scatter(self, send: torch.Tensor, recv: torch.Tensor, op: int = lib.REDUCE_SUM,
                       stream: int | None = None) -> torch.Tensor:
        assert send.numel() == recv.numel() * self.world
        lib.call("magma_reduce_scatter", send.data_ptr(), recv.data_ptr(), recv.numel(),
                 _DT[send.dtype], op, self.handle, _stream(send) if stream is None else stream)
        return recv

    def all_gather(self, send: torch.Tensor, recv: torch.Tensor,
                   stream: int | None = None) -> torch.Tensor:
        assert recv.numel() == send.numel() * self.world
        lib.call("magma_all_gather", send.data_ptr(), recv.data_ptr(), send.numel(),
                 _DT[send.dtype], self.handle, _stream(send) if stream is None else stream)
        return recv

    def destroy(self) -> None:
        if self.handle:
            lib.call("magma_comm_destroy", self.handle)
            self.handle = C.c_void_p()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


class _Event:
    """An event of the C ABI (no timing)."""

    def __init__(self):
        self.h = C.c_void_p()
        lib.call("magma_event_create", C.byref(self.h), 0)

    def record(self, stream: int) -> None:
        lib.call("magma_event_record", self.h, stream)

    def wait(self, stream: int) -> None:
        lib.call("magma_stream_wait_event", stream, self.h)

    def __del__(self):
        try:
            if self.h:
                lib.call("magma_event_destroy", self.h)
        except Exception:
            pass


class GradSync:
    """Sum all-reduce of a flat gradient arena in buckets; returns 1/world.

    ``bucket_bytes`` bounds each collective (large buckets amortise launch
    latency; NVSwitch gives every peer full bandwidth, so link count does not
    enter the choice). CUDA gradients go through ``comm`` (a ``Comm``; made
    from the default process group on first use); CPU gradients through
    torch.distributed (gloo), synchronously.
    """

    def __init__(self, group=None, bucket_bytes: int = 256 << 20, comm: Comm | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.bucket_bytes = bucket_bytes
        self.comm = comm
        self._stream = None
        self._ready = self._done = None
        self._pending = False

    def _buckets(self, grads: torch.Tensor):
        flat = grads.view(-1)
        per = max(1, self.bucket_bytes // flat.element_size())
        for start in range(0, flat.numel(), per):
            yield flat[start:start + per]

    def _cuda_setup(self, device) -> None:
        if self.comm is None:
            self.comm = Comm.from_process_group(self.group)
        if self._stream is None:
            self._stream = torch.cuda.Stream(device)
            self._ready, self._done = _Event(), _Event()

    def __call__(self, grads: torch.Tensor) -> float:
        """Blocking form: sums grads over the ranks in place on the current stream."""
        if self.world == 1:
            return 1.0
        if not grads.is_cuda:
            for b in self._buckets(grads):
                dist.all_reduce(b, op=dist.ReduceOp.SUM, group=self.group)
            return 1.0 / self.world
        self._cuda_setup(grads.device)
        for b in self._buckets(grads):
            self.comm.allreduce(b)
        return 1.0 / self.world

    def launch(self, grads: torch.Tensor) -> None:
        """Starts the sum all-reduce of one finished gradient range. On CUDA it
        runs on a communication stream ordered after the work queued so far on
        the current stream, so the next backward segment overlaps it; finish()
        joins. Every rank must launch the same ranges in the same order. (CPU
        tensors: done synchronously.)"""
        if self.world == 1:
            return
        if not grads.is_cuda:
            for b in self._buckets(grads):
                dist.all_reduce(b, op=dist.ReduceOp.SUM, group=self.group)
            return
        self._cuda_setup(grads.device)
        cur = _stream(grads)
        self._ready.record(cur)
        self._ready.wait(self._stream.cuda_stream)
        for b in self._buckets(grads):
            self.comm.allreduce(b, stream=self._stream.cuda_stream)
        self._pending = True

    def finish(self) -> float:
        """Makes the current stream wait for every launched all-reduce and
        returns the 1/world scale for Adam."""
        if self.world == 1:
            return 1.0
        if self._pending:
            self._done.record(self._stream.cuda_stream)
            self._done.wait(torch.cuda.current_stream(self._stream.device).cuda_stream)
            self._pending = False
        return 1.0 / self.world

    def close(self) -> None:
        """Destroys the communicator (call before destroy_process_group)."""
        if self.comm is not None:
            self.comm.destroy()
            self.comm = None


class ShardSync:
    """The exchange of sharded data parallelism (ZeRO stage 1) over a Comm:
    each finished gradient range is reduce-scattered in place (rank r keeps the
    sum of block r of the range; the range's length must split evenly), on a
    communication stream that overlaps the rest of the backward like
    GradSync's all-reduce; after the sharded Adam step, gather_range
    all-gathers each range of the updated parameters in place."""

    def __init__(self, comm: Comm):
        self.comm, self.world, self.rank = comm, comm.world, comm.rank
        self._stream = None
        self._ready = self._done = None
        self._pending = False

    def owned(self, lo: int, hi: int) -> tuple[int, int]:
        """This rank's slice [a, b) of the arena range [lo, hi)."""
        n = hi - lo
        if n % (4 * self.world):
            raise ValueError(f"range of {n} elements does not split into {self.world} slices "
                             "of whole 16-byte groups")
        per = n // self.world
        return lo + self.rank * per, lo + (self.rank + 1) * per

    def launch(self, grads: torch.Tensor) -> None:
        """Reduce-scatters one finished range (a 1-D view of the arena) in place."""
        if self._stream is None:
            self._stream = torch.cuda.Stream(grads.device)
            self._ready, self._done = _Event(), _Event()
        self._ready.record(_stream(grads))
        self._ready.wait(self._stream.cuda_stream)
        per = grads.numel() // self.world
        self.comm.reduce_scatter(grads, grads[self.rank * per:(self.rank + 1) * per],
                                 stream=self._stream.cuda_stream)
        self._pending = True

    def finish(self) -> float:
        if self._pending:
            self._done.record(self._stream.cuda_stream)
            self._done.wait(torch.cuda.current_stream(self._stream.device).cuda_stream)
            self._pending = False
        return 1.0 / self.world

    def gather_range(self, arena: torch.Tensor, lo: int, hi: int, stream: int | None = None):
        a, b = self.owned(lo, hi)
        self.comm.all_gather(arena[a:b], arena[lo:hi], stream=stream)


def shard_batch(global_tokens: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [rank*b, (rank+1)*b) of a [world*b, S] batch (DistributedSampler's
    contiguous split, Data.swift:151-230)."""
    b = global_tokens.shape[0] // world
    return global_tokens[rank * b:(rank + 1) * b]
