"""Session-memory helpers of the reference (mka/layers/session_memory.py) on B200.

causal_prefix_ema runs the stage-1 scan kernel (gate fixed to select L2);
repeat_retrieval_to_length keeps the reference's tensor semantics (it is a
view/copy utility; the fused forward never materialises it, the stage-1 kernel
reads L3 row min(t, T3 - 1) directly).
"""
from __future__ import annotations

import torch

from .. import ops


def causal_prefix_ema(x: torch.Tensor, beta: float = 0.9) -> torch.Tensor:
    """[B, T, D] -> [B, T, D]: L2[t] = beta * L2[t-1] + (1 - beta) * x[t], L2[-1] = 0
    (session_memory.py:6-22). Computed with an fp32 state; returned in x's dtype."""
    out = ops.causal_prefix_ema(x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16), beta)
    return out if x.dtype == torch.bfloat16 else out.to(x.dtype)


def repeat_retrieval_to_length(mem: torch.Tensor, target_len: int) -> torch.Tensor:
    """[B, T3, D] -> [B, T, D] by repeat / truncate / pad-with-last-row
    (session_memory.py:25-39)."""
    n = mem.size(1)
    if n == target_len:
        return mem
    idx = torch.clamp(torch.arange(target_len, device=mem.device), max=n - 1)
    return mem.index_select(1, idx)
