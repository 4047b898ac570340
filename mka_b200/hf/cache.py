"""Preallocated, in-place K/V cache for the decode path.

The reference concatenates the whole cache on every decode step
(torch.cat at mka/hf/attention.py:121-124 and mka/layers/fastmka.py:102-106), an
O(T) copy per token. A StaticKVCache holds one [B, Hkv, capacity, 128] bf16
buffer pair per attention layer; the K/V projection kernel writes the new
tokens straight into their slots and attention reads the valid prefix in place.
Pass it as `past_key_value` to HFFastMKAAttention.

With `carry_ema=True` the cache also keeps each layer's EMA (L2) state in
fp32 (that of x [Wk ; Wv]^T, [B, 2*Hkv*128], the space the layer's scan runs
in), so that the L2 memory continues across calls instead of restarting at
zero on every call as the reference does (session_memory.py:17-21): a decode
step then sees the same L2 as the reference's prefill of the whole sequence.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import torch
import torch.nn as nn


class StaticKVCache:
    def __init__(self, batch: int, num_kv_heads: int, capacity: int, num_layers: int = 1,
                 device: torch.device | str = "cuda", head_dim: int = 128, carry_ema: bool = False):
        self.batch = batch
        self.carry_ema = carry_ema
        self._ema: Dict[int, List[torch.Tensor]] = {}  # layer -> [state in, state out]
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

    def ema_buffers(self, module: nn.Module, d_model: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        """(state before this call, buffer for the state after it) of the layer;
        zero before the layer's first call."""
        i = self._index(module)
        if i not in self._ema:
            self._ema[i] = [torch.zeros((self.batch, d_model), dtype=torch.float32, device=device)
                            for _ in range(2)]
        return self._ema[i][0], self._ema[i][1]

    def commit_ema(self, module: nn.Module) -> None:
        """Makes the state written by the last call the next call's input."""
        bufs = self._ema[self._index(module)]
        bufs.reverse()

    def load_prefix(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Copies an existing [B, Hkv, T, 128] cache into slot `layer`."""
        t = k.shape[2]
        self.k[layer][:, :, :t].copy_(k)
        self.v[layer][:, :, :t].copy_(v)
        self.lengths[layer] = t
