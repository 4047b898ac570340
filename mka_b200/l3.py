"""L3 chunk recall: a bank of historical chunks and the retrieval that produces
the L3 memory R of the route blend.

The reference describes this tier and does not implement it:
mka/config/memory_hierarchy.py:1-10 ("L3 - DRAM (vectorized hash, chunk
recall): long-term retrieval / historical blocks") and lines 30-34
(`l3_dram_chunk_recall`, `l3_recall_top_r`: "top-R chunks per query"). Its
layers take R from the caller (mka/layers/fastmka.py:84-89,
mka/hf/attention.py:100-102). This module is the package's own form of that
description, with the bank resident in HBM:

  * a chunk is `chunk_len` consecutive hidden states of an earlier context;
    its key and its value are the chunk's mean (any [n_chunks, D] keys and
    values can be given instead);
  * the queries are the means of `block_len`-token blocks of the current
    hidden states; each block takes its `top_r` best chunks by dot product,
    weighted by softmax(scale * score), and every token of the block receives
    their weighted sum as its L3 row.

`R = store.recall(x)` is the `l3_memory` the patched attention accepts.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import ops


class L3ChunkStore:
    """A bank of n_chunks historical chunks: keys and values [n_chunks, D] bf16 on the GPU."""

    def __init__(self, keys: torch.Tensor, values: Optional[torch.Tensor] = None):
        values = keys if values is None else values
        if keys.dim() != 2 or keys.shape != values.shape:
            raise ValueError("keys and values must both be [n_chunks, D]")
        if not keys.is_cuda or keys.dtype != torch.bfloat16 or values.dtype != torch.bfloat16:
            raise ValueError("keys and values must be bf16 CUDA tensors")
        self.keys = keys.contiguous()
        self.values = values.contiguous()

    @property
    def n_chunks(self) -> int:
        return self.keys.shape[0]

    @classmethod
    def from_history(cls, hidden: torch.Tensor, chunk_len: int) -> "L3ChunkStore":
        """Chunks of `chunk_len` tokens of earlier hidden states ([T, D] or [B, T, D],
        each batch row chunked on its own); key = value = the chunk's mean."""
        h = hidden if hidden.dim() == 3 else hidden.unsqueeze(0)
        means = ops.l3_block_mean(h.contiguous(), chunk_len)
        return cls(means, means)

    def append(self, other: "L3ChunkStore") -> "L3ChunkStore":
        """The bank with another bank's chunks added after this one's."""
        return L3ChunkStore(torch.cat([self.keys, other.keys]), torch.cat([self.values, other.values]))

    def recall_with_indices(self, x: torch.Tensor, top_r: int = 8, block_len: int = 64,
                            scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(R [B, T, D] bf16, idx [B * nq, top_r] int32, w [B * nq, top_r] fp32) for x [B, T, D]."""
        if top_r < 1 or top_r > min(32, self.n_chunks):
            raise ValueError(f"top_r must be in 1..{min(32, self.n_chunks)}")
        return ops.l3_chunk_recall(x, self.keys, self.values, top_r, block_len, scale)

    def recall(self, x: torch.Tensor, top_r: int = 8, block_len: int = 64,
               scale: Optional[float] = None) -> torch.Tensor:
        """The L3 memory R [B, T, D] for x [B, T, D] (the `l3_memory` of the patched attention)."""
        return self.recall_with_indices(x, top_r, block_len, scale)[0]
