"""Synthetic token streams for benchmarks and tests.

Token ids are uniform over the vocabulary from a seeded generator (one
independent stream per rank).  ``PinnedBatchPool`` pre-generates a few
batches in page-locked host memory so a benchmark can measure the real
host->device input copy every step without paying for generation.

Reference parity: build_dummy_dataset (veomni/data/dummy_dataset.py:420).
"""

from __future__ import annotations

import torch


class SyntheticTokens:
    def __init__(self, vocab_size: int, batch: int, seq_len: int, seed: int = 0, rank: int = 0):
        self.vocab, self.batch, self.seq = vocab_size, batch, seq_len
        self.g = torch.Generator().manual_seed(seed * 7919 + rank)

    def __iter__(self):
        return self

    def __next__(self) -> torch.Tensor:
        return torch.randint(0, self.vocab, (self.batch, self.seq), generator=self.g, dtype=torch.int64)


class PinnedBatchPool:
    def __init__(self, vocab_size: int, batch: int, seq_len: int, n: int = 4, seed: int = 0, rank: int = 0):
        src = SyntheticTokens(vocab_size, batch, seq_len, seed, rank)
        pin = torch.cuda.is_available()
        self.batches = [next(src).pin_memory() if pin else next(src) for _ in range(n)]
        self.i = 0

    def __iter__(self):
        return self

    def __next__(self) -> torch.Tensor:
        b = self.batches[self.i % len(self.batches)]
        self.i += 1
        return b

    @property
    def bytes_per_batch(self) -> int:
        b = self.batches[0]
        return b.numel() * b.element_size()
