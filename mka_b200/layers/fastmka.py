"""FastMKAAttention on B200: the reference module's API (FastLM/MKA
mka/layers/fastmka.py:19-177) with every op running on the sm_100a kernels.

Same config fields, parameter names and shapes (wq, wk, wv, wo, router.0,
router.2), so reference state_dicts load unchanged; same forward signature and
return value (out, k_tot, v_tot, lam). Differences, all deliberate:
  * compute is bf16 with fp32 accumulation; outputs come back in x's dtype
  * head_dim must be 128; inference only (no dropout inside attention)
  * the reference's CUDA/SDPA dispatch flags (use_cuda_kernel, prefer_sdpa,
    use_fused_route_cuda) are accepted and ignored: there is one path
  * CPU tensors raise instead of falling back
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from .forward import fastmka_forward
from .prepared import PreparedWeights, prepare


@dataclass
class FastMKAConfig:
    """mka/layers/fastmka.py:19-31, plus the router width (default D/2, the
    reference's) and activation ("silu", the reference's, or "gelu")."""
    hidden_size: int
    num_heads: int
    use_l3: bool = True
    ema_beta: float = 0.9
    dropout_p: float = 0.0
    use_cuda_kernel: bool = True
    prefer_sdpa: bool = True
    use_fused_route_cuda: bool = False
    router_hidden: Optional[int] = None
    router_act: str = "silu"


class FastMKAAttention(nn.Module):
    """Route-fused MKA: L1 = x, L2 = causal prefix EMA, optional L3; lambda =
    softmax(MLP(q)); one K/V projection of sum(lambda_l L_l); one causal attention."""

    def __init__(self, cfg: FastMKAConfig):
        super().__init__()
        assert cfg.hidden_size % cfg.num_heads == 0
        self.cfg = cfg
        self.head_dim = cfg.hidden_size // cfg.num_heads
        d = cfg.hidden_size
        self.wq = nn.Linear(d, d, bias=False)
        self.wk = nn.Linear(d, d, bias=False)
        self.wv = nn.Linear(d, d, bias=False)
        self.wo = nn.Linear(d, d, bias=False)
        levels = 3 if cfg.use_l3 else 2
        r = cfg.router_hidden or d // 2
        act = nn.GELU() if cfg.router_act == "gelu" else nn.SiLU()
        self.router = nn.Sequential(nn.Linear(d, r), act, nn.Linear(r, levels))
        self.dropout = nn.Dropout(cfg.dropout_p)
        self._prep: Optional[PreparedWeights] = None

    def prepared(self, device: torch.device) -> PreparedWeights:
        self._prep = prepare(self.wq, self.wk, self.wv, self.wo, self.router, device, self._prep)
        return self._prep

    def forward_with_lse(self, x: torch.Tensor, l3_memory: Optional[torch.Tensor] = None,
                         kv_cache_k: Optional[torch.Tensor] = None, kv_cache_v: Optional[torch.Tensor] = None):
        """forward() plus the attention log-sum-exp [B, H, T] (fp32)."""
        if self.training and self.cfg.dropout_p > 0:
            raise NotImplementedError("the B200 path is forward-only (attention dropout is not implemented)")
        past = None
        if kv_cache_k is not None and kv_cache_v is not None:
            past = (kv_cache_k.to(torch.bfloat16), kv_cache_v.to(torch.bfloat16))
        with torch.no_grad():
            r = fastmka_forward(x, self.prepared(x.device), self.cfg.num_heads, self.cfg.num_heads,
                                self.cfg.ema_beta, self.cfg.use_l3, l3_memory=l3_memory, past=past)
        dt = x.dtype
        return r["out"].to(dt), r["k"].to(dt), r["v"].to(dt), r["lam"].to(dt), r["lse"]

    def forward(self, x: torch.Tensor, l3_memory: Optional[torch.Tensor] = None,
                kv_cache_k: Optional[torch.Tensor] = None, kv_cache_v: Optional[torch.Tensor] = None):
        out, k_tot, v_tot, lam, _ = self.forward_with_lse(x, l3_memory, kv_cache_k, kv_cache_v)
        return out, k_tot, v_tot, lam
