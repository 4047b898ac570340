"""FastMKA attention forward on NVIDIA B200 (sm_100a).

Drop-in for the FastLM/MKA FastMKA hot path: the module API of
mka.layers.FastMKAAttention / mka.hf.HFFastMKAAttention, the self_attn patch of
mka.hf.patch and the op API of mka.cuda.ops, all running hand-written sm_100a
kernels from libfastmka_b200.so (include/fastmka_b200.h) through a C ABI.
"""
from .hf import HFFastMKAAttention, HFPatchConfig, StaticKVCache, apply_hf_attention_patch, parse_patch_config
from .layers import FastMKAAttention, FastMKAConfig, causal_prefix_ema, repeat_retrieval_to_length

__all__ = ["FastMKAAttention", "FastMKAConfig", "HFFastMKAAttention", "HFPatchConfig", "StaticKVCache",
           "apply_hf_attention_patch", "parse_patch_config", "causal_prefix_ema", "repeat_retrieval_to_length"]
