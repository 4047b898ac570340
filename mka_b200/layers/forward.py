"""The FastMKA forward on B200: five launches, no intermediate round trips
beyond what the data flow needs.

  1. qr_proj          q = x Wq^T (+bq) -> head-split [B,Hq,T,128] (+RoPE), and the
                      router hidden act(x (W1 Wq)^T + b1') reduced against W2 into
                      per-token gate logits, in the GEMM epilogue
  2. kv_proj          y = x [Wk ; Wv]^T (bf16, 2*Hkv*128 channels); with three
                      levels also y3 = L3 [Wk ; Wv]^T
  3. route_ema_blend  lam = softmax(logits + b2); K/V = lam0 y + lam1 EMA(y)
                      (+ lam2 y3) (+bias, RoPE on K) -> head-split K/V, written
                      straight into the K/V buffer after any cached prefix. This
                      is the reference's projection of lam0 x + lam1 EMA(x)
                      (+ lam2 L3) in the commuted order (EMA along tokens,
                      projection along channels; the gate sums to one)
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
    ema_state / ema_out: fp32 EMA state before this call's first token (None:
             zero, the reference's restart) and a buffer for the state after its
             last token, to carry the L2 memory across calls. The scan runs
             on x [Wk ; Wv]^T, so the state is that of EMA(y), [B, 2*Hkv*128].
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
    k_tot, v_tot, lam = _kv_levels(xb, logits, W, B, T, D, num_kv_heads, beta, rope, past, kv_out, past_len,
                                   kv_update, ema_state, ema_out, use_l3, l3_memory, mark, done)
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


def _kv_buffers(B, T, num_kv_heads, past, kv_out, past_len, device):
    """Where this call's K/V land: (k_target, v_target, t_offset, k_total, v_total);
    targets None means fresh [B, Hkv, T, 128] buffers made by the kernel wrapper."""
    if kv_out is not None:
        kc, vc = kv_out
        tp = int(past_len or 0)
        if tp + T > kc.shape[2]:
            raise RuntimeError("preallocated K/V cache is full")
        return kc, vc, tp, kc[:, :, : tp + T], vc[:, :, : tp + T]
    if past is not None:
        pk, pv = past
        tp = pk.shape[2]
        k_tot = torch.empty((B, num_kv_heads, tp + T, HEAD_DIM), dtype=torch.bfloat16, device=device)
        v_tot = torch.empty_like(k_tot)
        k_tot[:, :, :tp].copy_(pk)
        v_tot[:, :, :tp].copy_(pv)
        return k_tot, v_tot, tp, k_tot, v_tot
    return None, None, 0, None, None


def _finish_kv(k_new, v_new, k_tot, v_tot, kv_update):
    if k_tot is None:
        k_tot, v_tot = k_new, v_new
        if kv_update is not None:
            k_tot, v_tot = kv_update(k_tot, v_tot)
            if k_tot.dtype != torch.bfloat16 or v_tot.dtype != torch.bfloat16:
                raise RuntimeError("the K/V returned by kv_update must be bf16")
    return k_tot, v_tot


def project_l3(l3_memory: Optional[torch.Tensor], W: PreparedWeights, B: int, D: int, num_kv_heads: int,
               device) -> torch.Tensor:
    """y3 = L3 [Wk ; Wv]^T ([B, T3, 2*Hkv*128] bf16): the third memory level in
    the projected space. No memory means the reference's zero L3
    (hf/attention.py:100-102), projected to zero without a GEMM."""
    n = 2 * num_kv_heads * HEAD_DIM
    if l3_memory is None:
        return torch.zeros((B, 1, n), dtype=torch.bfloat16, device=device)
    l3 = l3_memory if l3_memory.dtype == torch.bfloat16 else l3_memory.to(torch.bfloat16)
    if l3.dim() != 3 or l3.shape[0] != B or l3.shape[2] != D:
        raise RuntimeError("l3_memory must be [B, T3, D]")
    t3 = l3.shape[1]
    return ops.gemm(l3.reshape(B * t3, D).contiguous(), W.w_kv).view(B, t3, n)


def _kv_levels(xb, logits, W, B, T, D, num_kv_heads, beta, rope, past, kv_out, past_len, kv_update,
               ema_state, ema_out, use_l3, l3_memory, mark, done):
    """y = x [Wk ; Wv]^T, then one scan over y's 2*Hkv*128 channels writes
    K/V = lam0 y + lam1 EMA(y) (+ lam2 y3) + bias (RoPE on K). Equal to
    projecting the blend lam0 x + lam1 EMA(x) (+ lam2 L3) (fastmka.py:83-99,
    hf/attention.py:97-111): the EMA runs along tokens and the projection along
    channels, and the gate sums to one; the scan then touches 2*Hkv*128
    channels instead of d_model."""
    kt, vt, tp, k_tot, v_tot = _kv_buffers(B, T, num_kv_heads, past, kv_out, past_len, xb.device)
    mark("kv_proj")
    y = ops.gemm(xb.view(B * T, D), W.w_kv)
    y3 = project_l3(l3_memory, W, B, D, num_kv_heads, xb.device) if use_l3 else None
    done()
    mark("route_ema_blend")
    k_new, v_new, lam = ops.route_ema_blend_kv(y, beta, logits, W.b2, B, T, num_kv_heads, bias=W.b_kv, rope=rope,
                                               k_out=kt, v_out=vt, t_offset=tp, ema_state=ema_state,
                                               ema_out=ema_out, y3=y3)
    done()
    k_tot, v_tot = _finish_kv(k_new, v_new, k_tot, v_tot, kv_update)
    return k_tot, v_tot, lam
