"""Sequence packing: several documents per row of seq_len tokens.

``pack_documents`` lays documents out back to back over ``rows x seq_len``
tokens and returns the token matrix with ``cu_seqlens``, the cumulative
document boundaries over the flattened tokens.  A document that does not fit
in the rest of a row continues in the next row as a new document (rows never
share a document, so attention and positions restart per row as well);
documents beyond the last row are dropped.  The model restarts rotary
positions and masks attention and the next-token loss at every boundary.

``PackedSyntheticTokens`` is the synthetic stream for packed training:
document lengths drawn uniformly from [min_len, max_len], tokens uniform
over the vocabulary, seeded per rank.

Reference parity: the packing collator and dynamic batching of
veomni/data/data_collator.py (cu_seqlens, position ids per document) and
veomni/data/dynamic_batching.py.
"""

from __future__ import annotations

import torch


def pack_documents(docs: list[torch.Tensor], rows: int, seq_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Token ids [rows, seq_len] and int32 cu_seqlens over the flattened tokens."""
    ids = torch.empty(rows * seq_len, dtype=torch.long)
    cu = [0]
    pos = 0
    total = rows * seq_len
    for d in docs:
        d = d.reshape(-1)
        i = 0
        while i < d.numel() and pos < total:
            room = seq_len - pos % seq_len
            n = min(room, d.numel() - i)
            ids[pos: pos + n] = d[i: i + n]
            pos += n
            i += n
            cu.append(pos)
        if pos >= total:
            break
    if pos < total:
        raise ValueError(f"documents fill {pos} of {total} tokens")
    return ids.view(rows, seq_len), torch.tensor(cu, dtype=torch.int32)


class PackedSyntheticTokens:
    """Infinite stream of (ids [rows, seq_len], cu_seqlens) with uniform-length synthetic documents."""

    def __init__(self, vocab_size: int, rows: int, seq_len: int, min_len: int = 64, max_len: int = 2048,
                 seed: int = 0, rank: int = 0):
        if not 1 <= min_len <= max_len:
            raise ValueError("need 1 <= min_len <= max_len")
        self.vocab_size, self.rows, self.seq_len = vocab_size, rows, seq_len
        self.min_len, self.max_len = min_len, max_len
        self.gen = torch.Generator().manual_seed(seed * 1000003 + rank)

    def __iter__(self):
        return self

    def __next__(self) -> tuple[torch.Tensor, torch.Tensor]:
        need, docs = self.rows * self.seq_len, []
        while need > 0:
            n = int(torch.randint(self.min_len, self.max_len + 1, (1,), generator=self.gen))
            docs.append(torch.randint(0, self.vocab_size, (n,), generator=self.gen))
            need -= n
        return pack_documents(docs, self.rows, self.seq_len)
