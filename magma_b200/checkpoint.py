"""Binary checkpoints in the reference's ``BinaryCheckpoint`` format.

Layout (``BinaryCheckpoint``, Sources/Core/Module.swift:4838-4992): every
integer is a little-endian uint32, every value a float32.

    "STCHKPT\\0"                       8-byte magic
    version                            1 or 2 (files are written as 2)
    parameter count, then per parameter:
        name length, name (UTF-8), rank, rank x dim, prod(dims) float32 values
    version 2 only: buffer count, then each buffer encoded like a parameter

Reading validates every length against the bytes left (a truncated or
corrupt file raises CheckpointError before anything is used), rejects ranks
above 64 and trailing bytes, and accepts version-1 files (no buffer section),
as the reference's loader does (Module.swift:4908-4992).

The trainer's optimiser state (Adam's m and v, and the step count) is not part
of the reference's model checkpoint; ``GPTTrainer.save_checkpoint`` writes it to
a second file in the same format (m and v as parameters named ``<name>.m`` and
``<name>.v``, the step as a rank-0 buffer), so one reader serves both.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b"STCHKPT\x00"
VERSION = 2
MAX_RANK = 64


class CheckpointError(RuntimeError):
    """A checkpoint that cannot be read: bad magic, unsupported version,
    truncated or corrupt contents, or a mismatch with what the caller expects."""


@dataclass
class Entry:
    """One named tensor of a checkpoint (F32 values, C order)."""
    name: str
    shape: tuple[int, ...]
    values: np.ndarray

    def __post_init__(self) -> None:
        self.shape = tuple(int(d) for d in self.shape)
        self.values = np.ascontiguousarray(self.values, dtype="<f4").reshape(-1)
        if self.values.size != math.prod(self.shape):
            raise CheckpointError(f"{self.name}: {self.values.size} values for shape {self.shape}")


def _u32(x: int) -> bytes:
    if not 0 <= x < 1 << 32:
        raise CheckpointError(f"value {x} does not fit the format's uint32 fields")
    return struct.pack("<I", x)


def encode(params: list[Entry], buffers: list[Entry] | None = None, version: int = VERSION) -> bytes:
    """The file contents for `params` (and, in version 2, `buffers`)."""
    if version not in (1, 2):
        raise CheckpointError(f"unsupported version {version}")
    if version == 1 and buffers:
        raise CheckpointError("version-1 files have no buffer section")
    out = [MAGIC, _u32(version)]

    def section(entries: list[Entry]) -> None:
        out.append(_u32(len(entries)))
        for e in entries:
            name = e.name.encode("utf-8")
            out.append(_u32(len(name)))
            out.append(name)
            out.append(_u32(len(e.shape)))
            out.extend(_u32(d) for d in e.shape)
            out.append(e.values.tobytes())

    section(params)
    if version == 2:
        section(buffers or [])
    return b"".join(out)


class _Reader:
    def __init__(self, data: bytes) -> None:
        self.data = memoryview(data)
        self.off = 0

    @property
    def remaining(self) -> int:
        return len(self.data) - self.off

    def take(self, n: int, what: str) -> memoryview:
        if n < 0 or n > self.remaining:
            raise CheckpointError(f"truncated file: need {n} bytes for {what} at offset "
                                  f"{self.off}, only {self.remaining} left")
        v = self.data[self.off:self.off + n]
        self.off += n
        return v

    def u32(self, what: str) -> int:
        return struct.unpack("<I", self.take(4, what))[0]

    def entry(self, kind: str, index: int) -> Entry:
        what = f"{kind} {index}"
        name = bytes(self.take(self.u32(f"{what} name length"), f"{what} name")).decode(
            "utf-8", errors="replace")
        rank = self.u32(f"{what} rank")
        if rank > MAX_RANK:
            raise CheckpointError(f"{what} has implausible rank {rank} (corrupt file?)")
        shape = tuple(self.u32(f"{what} shape") for _ in range(rank))
        count = math.prod(shape)
        if count * 4 > self.remaining:
            raise CheckpointError(f"truncated file: need {count * 4} bytes for {what} values at "
                                  f"offset {self.off}, only {self.remaining} left")
        values = np.frombuffer(self.take(4 * count, f"{what} values"), dtype="<f4").astype(
            np.float32)
        return Entry(name, shape, values)


def decode(data: bytes) -> tuple[int, list[Entry], list[Entry]]:
    """(version, parameters, buffers) of a checkpoint's bytes."""
    r = _Reader(data)
    if r.remaining < len(MAGIC) or bytes(r.take(len(MAGIC), "magic")) != MAGIC:
        raise CheckpointError("Invalid file format (bad magic number)")
    version = r.u32("version")
    if not 1 <= version <= VERSION:
        raise CheckpointError(f"incompatible checkpoint version {version}")
    params = [r.entry("parameter", i) for i in range(r.u32("parameter count"))]
    buffers = []
    if version >= 2:
        buffers = [r.entry("buffer", i) for i in range(r.u32("buffer count"))]
    if r.remaining != 0:
        raise CheckpointError(f"{r.remaining} unexpected trailing bytes")
    return version, params, buffers


def save(path: str | Path, params: list[Entry], buffers: list[Entry] | None = None,
         version: int = VERSION) -> None:
    """Writes a checkpoint file (atomically: a temporary file, then a rename)."""
    path = Path(path)
    tmp = path.with_name(path.name + ".tmp")
    tmp.write_bytes(encode(params, buffers, version))
    tmp.replace(path)


def load(path: str | Path) -> tuple[int, list[Entry], list[Entry]]:
    """(version, parameters, buffers) of a checkpoint file."""
    try:
        data = Path(path).read_bytes()
    except OSError as e:
        raise CheckpointError(f"cannot read {path}: {e}") from e
    return decode(data)


def match(entries: list[Entry], expected: list[tuple[str, tuple[int, ...]]], kind: str) -> None:
    """Checks count, order and shapes against the model's tensors (the
    reference matches by position and checks shapes, Module.swift:4932-4939)."""
    if len(entries) != len(expected):
        raise CheckpointError(f"{kind} count mismatch: model has {len(expected)}, "
                              f"checkpoint has {len(entries)}")
    for i, (e, (name, shape)) in enumerate(zip(entries, expected)):
        if tuple(e.shape) != tuple(shape):
            raise CheckpointError(f"{kind} {i} ({name}): checkpoint shape {e.shape}, model "
                                  f"shape {tuple(shape)}")
