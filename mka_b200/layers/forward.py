"""The FastMKA forward on B200: five launches, no intermediate round trips
beyond what the data flow needs.

  1. qr_proj          q = x Wq^T (+bq) -> head-split [B,Hq,T,128] (+RoPE), and the
                      router hidden act(x (W1 Wq)^T + b1') reduced against W2 into
                      per-token gate logits, in the GEMM epilogue
  2. route_ema_blend  lam = softmax(logits + b2); L2 = prefix EMA of x; fused
                      H = lam0 x + lam1 L2 (+ lam2 L3); H written once
  3. kv_proj          [K | V] = H [Wk ; Wv]^T (+bias) -> head-split K/V (+RoPE on K),
                      written straight into the K/V buffer after any cached prefix
  4. attention        tcgen05 causal flash attention (prefill) or split-KV decode
                      (one new token), output [B, T, Hq, 128] and LSE
  5. o_proj           out = O Wo^T (+bo)

Reference: mka/layers/fastmka.py:71-177 and mka/hf/attention.py:82-199.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch

from .. import ops
from .prepared import PreparedWeights

HEAD_DIM = ops.HEAD_DIM


def fastmka_forward(x: torch.Tensor, W: PreparedWeights, num_heads: int, num_kv_heads: int, beta: float,
                    use_l3: bool, l3_memory: Optional[torch.Tensor] = None,
                    past: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                    rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                    kv_out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                    past_len: Optional[int] = None, timers: Optional[list] = None,
                    kv_update: Optional[Callable[[torch.Tensor, torch.Tensor],
                                                 Tuple[torch.Tensor, torch.Tensor]]] = None,
                    ema_state: Optional[torch.Tensor] = None, ema_out: Optional[torch.Tensor] = None) -> dict:
    """Runs the layer on x [B, T, D] (any float dtype; computed in bf16).

    past:    (k, v) [B, Hkv, Tp, 128] cached keys/values; the returned k/v are
             cat(past, new) as in the reference (a fresh buffer).
    kv_out:  alternatively a preallocated (k, v) cache [B, Hkv, Tcap, 128] whose
             first `past_len` slots are valid; new K/V are written in place at
             [past_len, past_len + T) and the returned k/v are views of the
             valid prefix (no copy of the cache).
    timers:  if a list is given, (stage, start_event, end_event) CUDA event
             pairs recorded on the current stream around each launch are appended.
    kv_update: alternatively a callable given this call's new (k, v)
             [B, Hkv, T, 128] (post-RoPE) that returns the full (k, v) to attend
             to, e.g. a transformers Cache's update(k, v, layer_idx).
    ema_state / ema_out: fp32 [B, D] EMA state before this call's first token
             (None: zero, the reference's restart) and a buffer for the state
             after its last token, to carry the L2 memory across calls.
    Returns dict(out [B,T,D] bf16, k, v, lam [B,T,L] fp32, lse).
    """
    def mark(name):
        if timers is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        timers.append([name, ev, None])
        return ev

    def done():
        if timers is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            timers[-1][2] = ev

    if not x.is_cuda:
        raise RuntimeError("the B200 FastMKA forward needs CUDA tensors (there is no CPU fallback)")
    B, T, D = x.shape
    if D % num_heads != 0 or D // num_heads != HEAD_DIM:
        raise NotImplementedError(f"head_dim must be {HEAD_DIM} (got {D // num_heads})")
    xb = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
    xb = xb.contiguous()
    L = 3 if use_l3 else 2
    if W.levels != L:
        raise RuntimeError(f"router has {W.levels} outputs but the layer blends {L} levels")

    # 1. q (+ RoPE) and router logits
    mark("qr_proj")
    q, logits = ops.qr_proj(xb.view(B * T, D), W.w_qr, W.b_qr, B, T, num_heads, W.router_hidden, W.w2, L,
                            W.act, rope=rope)
    done()
    # 2. gate + EMA + blend
    l3 = None
    if use_l3:
        if l3_memory is None:
            l3 = torch.zeros((B, 1, D), dtype=torch.bfloat16, device=x.device)
        else:
            l3 = l3_memory if l3_memory.dtype == torch.bfloat16 else l3_memory.to(torch.bfloat16)
            if l3.shape[0] != B or l3.shape[2] != D:
                raise RuntimeError("l3_memory must be [B, T3, D]")
    mark("route_ema_blend")
    h, lam = ops.route_ema_blend(xb, beta, logits=logits, b2=W.b2, levels=L, l3=l3, ema_state=ema_state,
                                 ema_out=ema_out)
    done()
    mark("kv_proj")
    # 3. K/V of the fused memory
    if kv_out is not None:
        kc, vc = kv_out
        tp = int(past_len or 0)
        if tp + T > kc.shape[2]:
            raise RuntimeError("preallocated K/V cache is full")
        ops.kv_proj(h.view(B * T, D), W.w_kv, W.b_kv, B, T, num_kv_heads, rope=rope, k_out=kc, v_out=vc,
                    t_offset=tp)
        k_tot, v_tot = kc[:, :, : tp + T], vc[:, :, : tp + T]
    elif past is not None:
        pk, pv = past
        tp = pk.shape[2]
        k_tot = torch.empty((B, num_kv_heads, tp + T, HEAD_DIM), dtype=torch.bfloat16, device=x.device)
        v_tot = torch.empty_like(k_tot)
        k_tot[:, :, :tp].copy_(pk)
        v_tot[:, :, :tp].copy_(pv)
        ops.kv_proj(h.view(B * T, D), W.w_kv, W.b_kv, B, T, num_kv_heads, rope=rope, k_out=k_tot, v_out=v_tot,
                    t_offset=tp)
    else:
        k_tot, v_tot = ops.kv_proj(h.view(B * T, D), W.w_kv, W.b_kv, B, T, num_kv_heads, rope=rope)
        if kv_update is not None:
            k_tot, v_tot = kv_update(k_tot, v_tot)
            if k_tot.dtype != torch.bfloat16 or v_tot.dtype != torch.bfloat16:
                raise RuntimeError("the K/V returned by kv_update must be bf16")
    done()
    # 4. attention
    mark("attention")
    if T == 1 and k_tot.shape[2] > 1:
        o, lse = ops.attn_decode(q, k_tot, v_tot)
        lse = lse.unsqueeze(-1)
    else:
        o, lse = ops.attn_prefill(q, k_tot, v_tot, causal=True)
    done()
    # 5. output projection
    mark("o_proj")
    out = ops.gemm(o.view(B * T, num_heads * HEAD_DIM), W.w_o, W.b_o).view(B, T, D)
    done()
    return {"out": out, "k": k_tot, "v": v_tot, "lam": lam, "lse": lse, "q": q}
