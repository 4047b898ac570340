"""Preallocated, in-place K/V cache for the decode path.

The reference concatenates the whole cache on every decode step
(torch.cat at mka/hf/attention.py:121-124 and mka/layers/fastmka.py:102-106), an
O(T) copy per token. A StaticKVCache holds one [B, Hkv, capacity, 128] bf16
buffer pair per attention layer; the K/V projection kernel writes the new
tokens straight into their slots and attention reads the valid prefix in place.
Pass it as `past_key_value` to HFFastMKAAttention.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import torch
import torch.nn as nn


class StaticKVCache:
    def __init__(self, batch: int, num_kv_heads: int, capacity: int, num_layers: int = 1,
                 device: torch.device | str = "cuda", head_dim: int = 128):
        self.batch = batch
        self.num_kv_heads = num_kv_heads
        self.capacity = capacity
        shape = (batch, num_kv_heads, capacity, head_dim)
        self.k: List[torch.Tensor] = [torch.empty(shape, dtype=torch.bfloat16, device=device) for _ in range(num_layers)]
        self.v: List[torch.Tensor] = [torch.empty(shape, dtype=torch.bfloat16, device=device) for _ in range(num_layers)]
        self.lengths: List[int] = [0] * num_layers
        self._slot: Dict[int, int] = {}

    def _index(self, module: nn.Module) -> int:
        key = id(module)
        if key not in self._slot:
            if len(self._slot) >= len(self.k):
                raise RuntimeError("StaticKVCache has fewer layers than the model uses")
            self._slot[key] = len(self._slot)
        return self._slot[key]

    def layer(self, module: nn.Module) -> Tuple[torch.Tensor, torch.Tensor]:
        i = self._index(module)
        return self.k[i], self.v[i]

    def length(self, module: nn.Module) -> int:
        return self.lengths[self._index(module)]

    def advance(self, module: nn.Module, n: int) -> None:
        i = self._index(module)
        if self.lengths[i] + n > self.capacity:
            raise RuntimeError("StaticKVCache capacity exceeded")
        self.lengths[i] += n

    def load_prefix(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Copies an existing [B, Hkv, T, 128] cache into slot `layer`."""
        t = k.shape[2]
        self.k[layer][:, :, :t].copy_(k)
        self.v[layer][:, :, :t].copy_(v)
        self.lengths[layer] = t
