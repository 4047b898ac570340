"""HFFastMKAAttention on B200: drop-in for the reference HF wrapper
(FastLM/MKA mka/hf/attention.py:36-199) with every op on the sm_100a kernels.

Same constructor (original_attn, use_l3, ema_beta, use_cuda_kernel, prefer_sdpa),
same reused projections (q_proj/k_proj/v_proj/o_proj), same router parameters
(router.0 / router.2, hidden D/2, SiLU), same forward signature and 3-tuple
return (attn_output, None, present). Behaviour follows the reference: RoPE is
applied when the wrapped module exposes `rotary_emb` (position_embeddings when
given, else rotary_emb(x, position_ids)); a tuple past_key_value is
concatenated and returned as `present` (post-RoPE k/v, [B, Hkv, T, Dh]) when
use_cache is set; GQA heads share K/V without materialising _repeat_kv.

Extensions: `l3_memory` ([B, T3, D]) feeds a per-position L3 level when
use_l3 is set (the reference always blends zeros, hf/attention.py:100-102);
the head counts are read from the wrapped module's config when the module no
longer carries them (transformers >= 4.48); a `StaticKVCache` passed as
past_key_value is written in place instead of concatenated; a transformers
Cache object (past_key_values of transformers >= 4.48: anything with
update(k, v, layer_idx)) receives the new post-RoPE k/v through its own
update and the layer attends to what it returns; `return_present=False`
gives the two-value return (attn_output, attn_weights) that the decoder
layers of transformers >= 4.48 unpack, and with it RoPE follows that
version's contract (position_embeddings from the model, no rotary_emb on the
module). Additive masks are not supported
(causal only): with the default sdpa attention implementation transformers
passes no mask for unpadded prefill and cached decode.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from ..layers.forward import fastmka_forward
from ..layers.prepared import PreparedWeights, prepare
from .cache import StaticKVCache


def _attr(mod: nn.Module, name: str, cfg_name: str, default=None):
    v = getattr(mod, name, None)
    if v is None:
        cfg = getattr(mod, "config", None)
        v = getattr(cfg, cfg_name, None) if cfg is not None else None
    return default if v is None else v


class HFFastMKAAttention(nn.Module):
    def __init__(self, original_attn: nn.Module, use_l3: bool = False, ema_beta: float = 0.9,
                 use_cuda_kernel: bool = True, prefer_sdpa: bool = True, return_present: bool = True):
        super().__init__()
        self.return_present = return_present
        self.layer_idx = getattr(original_attn, "layer_idx", None)
        self.original_attn = original_attn
        self.use_l3 = use_l3
        self.ema_beta = ema_beta
        self.use_cuda_kernel = use_cuda_kernel
        self.prefer_sdpa = prefer_sdpa

        self.hidden_size = _attr(original_attn, "hidden_size", "hidden_size")
        self.num_heads = _attr(original_attn, "num_heads", "num_attention_heads")
        if self.hidden_size is None or self.num_heads is None:
            raise ValueError("cannot determine hidden_size / num_heads of the wrapped attention module")
        self.head_dim = self.hidden_size // self.num_heads
        self.num_key_value_heads = _attr(original_attn, "num_key_value_heads", "num_key_value_heads", self.num_heads)
        self.num_key_value_groups = self.num_heads // self.num_key_value_heads

        self.q_proj = original_attn.q_proj
        self.k_proj = original_attn.k_proj
        self.v_proj = original_attn.v_proj
        self.o_proj = original_attn.o_proj
        self.rotary_emb = getattr(original_attn, "rotary_emb", None)
        self.attention_dropout = float(getattr(original_attn, "attention_dropout", 0.0))

        levels = 3 if use_l3 else 2
        self.router = nn.Sequential(
            nn.Linear(self.hidden_size, self.hidden_size // 2),
            nn.SiLU(),
            nn.Linear(self.hidden_size // 2, levels),
        )
        self._prep: Optional[PreparedWeights] = None

    def prepared(self, device: torch.device) -> PreparedWeights:
        self._prep = prepare(self.q_proj, self.k_proj, self.v_proj, self.o_proj, self.router, device, self._prep)
        return self._prep

    def forward_with_lse(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                         position_ids: Optional[torch.Tensor] = None,
                         past_key_value=None, output_attentions: bool = False, use_cache: bool = False,
                         cache_position: Optional[torch.Tensor] = None,
                         position_embeddings: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                         l3_memory: Optional[torch.Tensor] = None, **kwargs):
        if output_attentions:
            raise NotImplementedError("output_attentions is not supported by the fused B200 path")
        if attention_mask is not None:
            raise NotImplementedError("additive attention masks are not supported (causal only); pass None")
        if past_key_value is None:
            past_key_value = kwargs.get("past_key_values")
        rope = None
        if self.rotary_emb is not None:
            if position_embeddings is not None:
                rope = position_embeddings
            else:
                rope = self.rotary_emb(hidden_states, position_ids)
        elif not self.return_present and position_embeddings is not None:
            # transformers >= 4.48: the model computes (cos, sin) once and the
            # attention modules no longer carry rotary_emb
            rope = position_embeddings
        dt = hidden_states.dtype
        W = self.prepared(hidden_states.device)
        with torch.no_grad():
            if _is_hf_cache(past_key_value):
                if self.layer_idx is None:
                    raise RuntimeError("a transformers Cache needs the wrapped attention's layer_idx")
                cache, idx = past_key_value, self.layer_idx
                r = fastmka_forward(hidden_states, W, self.num_heads, self.num_key_value_heads, self.ema_beta,
                                    self.use_l3, l3_memory=l3_memory, rope=rope,
                                    kv_update=lambda k, v: cache.update(k, v, idx))
                present = None  # the Cache object holds them
            elif isinstance(past_key_value, StaticKVCache):
                cache = past_key_value
                kc, vc = cache.layer(self)
                ema_in = ema_out = None
                if cache.carry_ema:
                    # the state of EMA(x [Wk ; Wv]^T), the space the layer's scan runs in
                    width = 2 * self.num_key_value_heads * self.head_dim
                    ema_in, ema_out = cache.ema_buffers(self, width, hidden_states.device)
                r = fastmka_forward(hidden_states, W, self.num_heads, self.num_key_value_heads, self.ema_beta,
                                    self.use_l3, l3_memory=l3_memory, rope=rope, kv_out=(kc, vc),
                                    past_len=cache.length(self), ema_state=ema_in, ema_out=ema_out)
                cache.advance(self, hidden_states.shape[1])
                if cache.carry_ema:
                    cache.commit_ema(self)
                present = (r["k"], r["v"]) if use_cache else None
            else:
                past = None
                if past_key_value is not None:
                    pk, pv = past_key_value
                    past = (pk.to(torch.bfloat16), pv.to(torch.bfloat16))
                r = fastmka_forward(hidden_states, W, self.num_heads, self.num_key_value_heads, self.ema_beta,
                                    self.use_l3, l3_memory=l3_memory, past=past, rope=rope)
                present = (r["k"].to(dt), r["v"].to(dt)) if use_cache else None
        return r["out"].to(dt), None, present, r["lse"], r["lam"]

    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None, past_key_value=None,
                output_attentions: bool = False, use_cache: bool = False,
                cache_position: Optional[torch.Tensor] = None,
                position_embeddings: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, **kwargs):
        out, w, present, _, _ = self.forward_with_lse(hidden_states, attention_mask, position_ids, past_key_value,
                                                      output_attentions, use_cache, cache_position,
                                                      position_embeddings, **kwargs)
        if not self.return_present:
            return out, w
        return out, w, present


def _is_hf_cache(obj) -> bool:
    """A transformers Cache (DynamicCache, StaticCache, ...): has update(k, v, layer_idx)."""
    return (obj is not None and not isinstance(obj, (tuple, list, StaticKVCache))
            and callable(getattr(obj, "update", None)))
