"""The feed-forward block around the patched self_attn, fused (optional).

The reference patches only self_attn (mka/hf/patch.py:30-48); the transformers
MLP of each decoder layer (LlamaMLP / Qwen2MLP / MistralMLP: down_proj(
act_fn(gate_proj(x)) * up_proj(x)) with act_fn = SiLU) then runs as three cuBLAS
GEMMs and two elementwise kernels, which write and re-read the two [tokens, I]
intermediates. `FusedSwiGLUMLP` computes silu(gate) * up in the epilogue of one
GEMM over the interleaved [gate ; up] weight (fmka_gemm_bf16_swiglu) and
down_proj with the package's GEMM, so each layer's feed-forward reads x once
and writes only the [tokens, I] product. Parameter names stay those of the
wrapped module (gate_proj / up_proj / down_proj), so state_dicts load
unchanged. `apply_mlp_fusion` installs it in every decoder layer whose MLP has
that form. `SiLUMulMLP` keeps transformers' three GEMMs and only fuses the
activation and the product into one pass (`apply_mlp_fusion(mode="silu_mul")`).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from .. import ops
from .patch import _iter_layers


def _is_silu(act) -> bool:
    return isinstance(act, nn.SiLU) or type(act).__name__ in ("SiLU", "SiLUActivation")


class FusedSwiGLUMLP(nn.Module):
    """Drop-in for a gated SiLU MLP with gate_proj / up_proj / down_proj Linears."""

    def __init__(self, mlp: nn.Module):
        super().__init__()
        self.gate_proj = mlp.gate_proj
        self.up_proj = mlp.up_proj
        self.down_proj = mlp.down_proj
        if self.gate_proj.out_features % 128:
            raise ValueError("FusedSwiGLUMLP: the intermediate size must be a multiple of 128")
        self._packed: Optional[Tuple[tuple, torch.Tensor, Optional[torch.Tensor], torch.Tensor]] = None

    def _weights(self, device: torch.device):
        ts = (self.gate_proj.weight, self.up_proj.weight, self.gate_proj.bias, self.up_proj.bias,
              self.down_proj.weight)
        key = tuple((t.data_ptr(), t._version, t.device) if t is not None else None for t in ts) + (device,)
        if self._packed is None or self._packed[0] != key:
            with torch.no_grad():
                bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16)  # noqa: E731
                w_gu = ops.interleave_gate_up(bf(self.gate_proj.weight), bf(self.up_proj.weight))
                b_gu = None
                if self.gate_proj.bias is not None or self.up_proj.bias is not None:
                    zg = torch.zeros(self.gate_proj.out_features, device=device)
                    bg = self.gate_proj.bias.detach().float().to(device) if self.gate_proj.bias is not None else zg
                    bu = self.up_proj.bias.detach().float().to(device) if self.up_proj.bias is not None else zg
                    b_gu = ops.interleave_gate_up(bg, bu)
                w_down = bf(self.down_proj.weight).contiguous()
            self._packed = (key, w_gu, b_gu, w_down)
        return self._packed[1:]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w_gu, b_gu, w_down = self._weights(x.device)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = x2.contiguous()
        with torch.no_grad():
            h = ops.gemm_swiglu(x2, w_gu, b_gu)
            out = ops.gemm(h, w_down, self.down_proj.bias)
        return out.view(*shape[:-1], out.shape[-1]).to(x.dtype)


class SiLUMulMLP(nn.Module):
    """Drop-in for a gated SiLU MLP that keeps its three GEMMs (the wrapped
    Linears, cuBLAS through torch) and replaces act_fn(gate) * up, two
    elementwise kernels over the [tokens, I] intermediates, by one pass
    (ops.silu_mul, written over the gate output). Same parameter names."""

    def __init__(self, mlp: nn.Module):
        super().__init__()
        self.gate_proj = mlp.gate_proj
        self.up_proj = mlp.up_proj
        self.down_proj = mlp.down_proj

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        g = self.gate_proj(x)
        u = self.up_proj(x)
        if g.dtype != torch.bfloat16:
            raise RuntimeError("SiLUMulMLP needs a bf16 model")
        with torch.no_grad():
            h = ops.silu_mul(g.contiguous(), u.contiguous(), out=g if g.is_contiguous() else None)
        return self.down_proj(h)


def apply_mlp_fusion(model: nn.Module, verbose: bool = False, mode: str = "swiglu") -> int:
    """Replaces every decoder layer's gated SiLU MLP, with FusedSwiGLUMLP (mode
    "swiglu": gate/up GEMM with the SiLU-product epilogue) or SiLUMulMLP (mode
    "silu_mul": transformers' GEMMs, one-pass SiLU product); returns the number
    of layers changed (inference: no autograd through it)."""
    if mode not in ("swiglu", "silu_mul"):
        raise ValueError("mode must be 'swiglu' or 'silu_mul'")
    fused = 0
    for layer in _iter_layers(model):
        mlp = getattr(layer, "mlp", None)
        if mlp is None or isinstance(mlp, (FusedSwiGLUMLP, SiLUMulMLP)):
            continue
        if not all(hasattr(mlp, n) for n in ("gate_proj", "up_proj", "down_proj")):
            continue
        if not _is_silu(getattr(mlp, "act_fn", None)):
            continue
        if mode == "swiglu":
            if mlp.gate_proj.out_features % 128:
                continue
            layer.mlp = FusedSwiGLUMLP(mlp)
        else:
            if mlp.gate_proj.weight.dtype != torch.bfloat16 or mlp.gate_proj.out_features % 8:
                continue
            layer.mlp = SiLUMulMLP(mlp)
        fused += 1
    if verbose:
        print(f"[MKA patch] fused MLP layers: {fused}")
    return fused
