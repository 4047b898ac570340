"""Device-side weight layouts for the fused FastMKA kernels, rebuilt only when a
parameter changes (tracked through each parameter's storage pointer and version
counter).

  w_qr = [Wq ; W1 Wq]   the Q projection stacked with the router's first layer
                        folded through Wq: router(q) = W2 act(W1 (Wq x + bq) + b1) + b2
                        = W2 act((W1 Wq) x + (W1 bq + b1)) + b2, so one GEMM over x
                        yields q and the router hidden state (folded in fp32)
  w_kv = [Wk ; Wv]      one GEMM for K and V of the fused memory
  w_o                   output projection
Router activation: nn.SiLU (the reference default, mka/layers/fastmka.py:55-59,
mka/hf/attention.py:71-76) or exact-erf nn.GELU (the MKAFullAttention router,
mka/layers/mka_full.py:34-38, and the single-layer fp32 configuration).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from .. import ops


@dataclass
class PreparedWeights:
    key: tuple
    w_qr: torch.Tensor            # bf16 [Hq*128 + R, D]
    b_qr: Optional[torch.Tensor]  # fp32 [Hq*128 + R]
    w2: torch.Tensor              # fp32 [L, R]
    b2: Optional[torch.Tensor]    # fp32 [L]
    router_hidden: int
    levels: int
    act: int
    w_kv: torch.Tensor            # bf16 [2*Hkv*128, D]
    b_kv: Optional[torch.Tensor]  # fp32 [2*Hkv*128]
    w_o: torch.Tensor             # bf16 [D, Hq*128]
    b_o: Optional[torch.Tensor]   # fp32 [D]


def router_act_code(router: nn.Sequential) -> int:
    if len(router) != 3 or not isinstance(router[0], nn.Linear) or not isinstance(router[2], nn.Linear):
        raise NotImplementedError("router must be Sequential(Linear, activation, Linear)")
    a = router[1]
    if isinstance(a, nn.SiLU):
        return ops.ACT_SILU
    if isinstance(a, nn.GELU) and getattr(a, "approximate", "none") == "none":
        return ops.ACT_GELU
    raise NotImplementedError(f"router activation {type(a).__name__} is not supported (SiLU or GELU)")


def _key(tensors) -> tuple:
    return tuple((t.data_ptr(), t._version, t.device) if t is not None else None for t in tensors)


def prepare(wq: nn.Linear, wk: nn.Linear, wv: nn.Linear, wo: nn.Linear, router: nn.Sequential,
            device: torch.device, cached: Optional[PreparedWeights] = None) -> PreparedWeights:
    tensors = [wq.weight, wq.bias, wk.weight, wk.bias, wv.weight, wv.bias, wo.weight, wo.bias,
               router[0].weight, router[0].bias, router[2].weight, router[2].bias]
    act = router_act_code(router)
    key = _key(tensors) + (act, device)
    if cached is not None and cached.key == key:
        return cached
    with torch.no_grad():
        f32 = lambda t: None if t is None else t.detach().to(device=device, dtype=torch.float32)  # noqa: E731
        Wq, bq = f32(wq.weight), f32(wq.bias)
        W1, b1 = f32(router[0].weight), f32(router[0].bias)
        W1q = W1 @ Wq
        b1q = b1.clone() if b1 is not None else torch.zeros(W1.shape[0], device=device)
        if bq is not None:
            b1q += W1 @ bq
        w_qr = torch.cat([Wq, W1q], 0).to(torch.bfloat16).contiguous()
        b_qr = torch.cat([bq if bq is not None else torch.zeros(Wq.shape[0], device=device), b1q]).contiguous()
        w_kv = torch.cat([f32(wk.weight), f32(wv.weight)], 0).to(torch.bfloat16).contiguous()
        b_kv = None
        if wk.bias is not None or wv.bias is not None:
            bk = f32(wk.bias) if wk.bias is not None else torch.zeros(wk.weight.shape[0], device=device)
            bv = f32(wv.bias) if wv.bias is not None else torch.zeros(wv.weight.shape[0], device=device)
            b_kv = torch.cat([bk, bv]).contiguous()
        return PreparedWeights(
            key=key, w_qr=w_qr, b_qr=b_qr, w2=f32(router[2].weight).contiguous(), b2=f32(router[2].bias),
            router_hidden=W1.shape[0], levels=router[2].weight.shape[0], act=act, w_kv=w_kv, b_kv=b_kv,
            w_o=f32(wo.weight).to(torch.bfloat16).contiguous(), b_o=f32(wo.bias))
