"""The RMSNorm of the decoder layers around the patched self_attn, in one kernel
(optional).

The reference patches only self_attn (mka/hf/patch.py:30-48); each decoder
layer's input_layernorm and post_attention_layernorm then run transformers'
LlamaRMSNorm / Qwen2RMSNorm: a chain of elementwise kernels with fp32
intermediates (for a 65536 x 4096 bf16 input about 8 GB of memory traffic per
norm). `FusedRMSNorm` computes the same thing in one pass (fmka_rmsnorm_bf16:
one read of x, one write of y) with the module's roundings, keeps the parameter
name `weight`, so state_dicts load unchanged, and `apply_norm_fusion` installs
it for every RMSNorm of a bf16 model. Its input must be a bf16 CUDA tensor.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops


def _is_rmsnorm(mod: nn.Module) -> bool:
    return (type(mod).__name__.endswith("RMSNorm") and isinstance(getattr(mod, "weight", None), torch.Tensor)
            and mod.weight.dim() == 1 and hasattr(mod, "variance_epsilon"))


class FusedRMSNorm(nn.Module):
    """Drop-in for LlamaRMSNorm-style modules (weight, variance_epsilon) on bf16 input."""

    def __init__(self, norm: nn.Module):
        super().__init__()
        self.weight = norm.weight
        self.variance_epsilon = float(norm.variance_epsilon)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        w = self.weight if self.weight.dtype == torch.bfloat16 else self.weight.to(torch.bfloat16)
        return ops.rmsnorm(hidden_states, w.detach().contiguous(), self.variance_epsilon)

    def extra_repr(self) -> str:
        return f"{tuple(self.weight.shape)}, eps={self.variance_epsilon}"


def apply_norm_fusion(model: nn.Module) -> int:
    """Replaces every bf16 RMSNorm module of `model` (decoder-layer norms and the
    final norm) by FusedRMSNorm; returns how many were replaced."""
    targets = []
    for name, mod in model.named_modules():
        for cname, child in mod.named_children():
            if _is_rmsnorm(child) and not isinstance(child, FusedRMSNorm) and child.weight.dtype == torch.bfloat16:
                targets.append((mod, cname, child))
    for parent, cname, child in targets:
        setattr(parent, cname, FusedRMSNorm(child))
    return len(targets)
