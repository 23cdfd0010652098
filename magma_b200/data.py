"""Token loader: ``MemoryMappedTokenDataset`` (Sources/Core/Data.swift:1827-2000).

A token file is a flat array of little-endian uint16 token ids. It is mapped,
not read (numpy memmap over the file), so a corpus of any size costs only the
pages that batches touch. Sample i is (tokens[i : i+S], tokens[i+1 : i+S+1]);
there are tokenCount - S samples (Data.swift:1841-1845, 1905-1917). Batches
are [batch, S] int32 arrays of inputs and targets, in index order or a
seeded shuffle, and the iterator stops before a partial batch, as the
reference's TokenBatchIterator does (Data.swift:1948-1999). ``pinned_batches``
fills page-locked host tensors so the trainer's host-to-device copy of each
batch runs asynchronously.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np


class TokenDatasetError(RuntimeError):
    """A token file that is missing or too small for one sample."""


class MemoryMappedTokenDataset:
    def __init__(self, path: str | Path, sequence_length: int) -> None:
        if sequence_length <= 0:
            raise TokenDatasetError("sequence_length must be positive")
        p = Path(path)
        if not p.is_file():
            raise TokenDatasetError(f"token file not found: {p}")
        self.path = p
        self.sequence_length = int(sequence_length)
        nbytes = p.stat().st_size
        self.token_count = nbytes // 2
        if self.token_count <= self.sequence_length:
            raise TokenDatasetError(f"token file too small: expected at least "
                                    f"{self.sequence_length + 1} tokens, got {self.token_count}")
        self.tokens = np.memmap(p, dtype="<u2", mode="r", shape=(self.token_count,))

    def __len__(self) -> int:
        return max(0, self.token_count - self.sequence_length)

    @property
    def count(self) -> int:
        return len(self)

    def get_tokens(self, start: int, length: int) -> np.ndarray:
        if start < 0 or length < 0 or start + length > self.token_count:
            raise IndexError("token range out of bounds")
        return self.tokens[start:start + length].astype(np.int32)

    def get_sample(self, index: int) -> tuple[np.ndarray, np.ndarray]:
        if not 0 <= index < len(self):
            raise IndexError("sample index out of bounds")
        t = self.get_tokens(index, self.sequence_length + 1)
        return t[:-1], t[1:]

    def batch(self, indices) -> tuple[np.ndarray, np.ndarray]:
        """Inputs and targets [len(indices), S] (int32) of the given samples."""
        idx = np.asarray(indices, dtype=np.int64)
        if idx.size and (idx.min() < 0 or idx.max() >= len(self)):
            raise IndexError("sample index out of bounds")
        win = idx[:, None] + np.arange(self.sequence_length + 1, dtype=np.int64)[None, :]
        t = self.tokens[win].astype(np.int32)
        return t[:, :-1], t[:, 1:]

    def batches(self, batch_size: int, shuffle: bool = True, seed: int = 0):
        """Yields (inputs, targets) [batch_size, S] int32 over one epoch; the
        last partial batch is dropped."""
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        order = np.arange(len(self), dtype=np.int64)
        if shuffle:
            np.random.default_rng(seed).shuffle(order)
        for i in range(0, len(order) - batch_size + 1, batch_size):
            yield self.batch(order[i:i + batch_size])

    def pinned_batches(self, batch_size: int, shuffle: bool = True, seed: int = 0, slots: int = 2):
        """Like batches(), as page-locked torch int32 tensors from a ring of
        `slots` buffer pairs (a slot is reused `slots` batches later, so the
        consumer must have finished copying it by then)."""
        import torch

        S = self.sequence_length
        ring = [(torch.empty((batch_size, S), dtype=torch.int32).pin_memory(),
                 torch.empty((batch_size, S), dtype=torch.int32).pin_memory())
                for _ in range(slots)]
        for k, (x, y) in enumerate(self.batches(batch_size, shuffle, seed)):
            tx, ty = ring[k % slots]
            tx.numpy()[...] = x
            ty.numpy()[...] = y
            yield tx, ty


def write_token_file(path: str | Path, tokens) -> None:
    """Writes token ids (each < 65536) as the loader's little-endian uint16."""
    a = np.asarray(tokens)
    if a.size and (a.min() < 0 or a.max() > 0xFFFF):
        raise ValueError("token ids must fit in uint16")
    a.astype("<u2").tofile(str(path))
