"""The self_attn monkey patch of the reference (FastLM/MKA mka/hf/patch.py:11-65),
installing the B200 HFFastMKAAttention. Same config dataclass, same layer walk
(model.model.layers or model.transformer.h), same return value (patched count).

Beyond the reference: on transformers >= 4.48 the decoder layers unpack two
values from self_attn and pass a Cache object, so the installed modules return
(attn_output, attn_weights) and route their K/V through the Cache; on older
versions they keep the reference's three-value return with tuple caches."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch.nn as nn

from .attention import HFFastMKAAttention


def _two_value_attention_api() -> bool:
    """True when the installed transformers' decoder layers unpack (out, weights)."""
    try:
        import transformers
    except ImportError:
        return False
    parts = []
    for piece in transformers.__version__.split(".")[:2]:
        digits = "".join(ch for ch in piece if ch.isdigit())
        parts.append(int(digits) if digits else 0)
    return tuple(parts) >= (4, 48)


@dataclass
class HFPatchConfig:
    enabled: bool = True
    mode: str = "fastmka"  # fastmka | off
    use_l3: bool = False
    ema_beta: float = 0.9
    use_cuda_kernel: bool = True
    prefer_sdpa: bool = True
    verbose: bool = True


def _iter_layers(model: nn.Module):
    if hasattr(model, "model") and hasattr(model.model, "layers"):
        return model.model.layers
    if hasattr(model, "transformer") and hasattr(model.transformer, "h"):
        return model.transformer.h
    raise ValueError("Unsupported model layout: cannot find decoder layers.")


def apply_hf_attention_patch(model: nn.Module, cfg: HFPatchConfig) -> int:
    if not cfg.enabled or cfg.mode == "off":
        return 0
    patched = 0
    two_value = _two_value_attention_api()
    for layer in _iter_layers(model):
        if not hasattr(layer, "self_attn"):
            continue
        attn = layer.self_attn
        if not all(hasattr(attn, n) for n in ("q_proj", "k_proj", "v_proj", "o_proj")):
            continue
        layer.self_attn = HFFastMKAAttention(attn, use_l3=cfg.use_l3, ema_beta=cfg.ema_beta,
                                             use_cuda_kernel=cfg.use_cuda_kernel, prefer_sdpa=cfg.prefer_sdpa,
                                             return_present=not two_value)
        patched += 1
    if cfg.verbose:
        print(f"[MKA patch] patched self_attn layers: {patched}")
    return patched


def parse_patch_config(raw: dict[str, Any]) -> HFPatchConfig:
    return HFPatchConfig(
        enabled=bool(raw.get("enabled", True)),
        mode=str(raw.get("mode", "fastmka")),
        use_l3=bool(raw.get("use_l3", False)),
        ema_beta=float(raw.get("ema_beta", 0.9)),
        use_cuda_kernel=bool(raw.get("use_cuda_kernel", True)),
        prefer_sdpa=bool(raw.get("prefer_sdpa", True)),
        verbose=bool(raw.get("verbose", True)),
    )
