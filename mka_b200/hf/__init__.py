from .attention import HFFastMKAAttention
from .cache import StaticKVCache
from .patch import HFPatchConfig, apply_hf_attention_patch, parse_patch_config

__all__ = ["HFFastMKAAttention", "StaticKVCache", "HFPatchConfig", "apply_hf_attention_patch", "parse_patch_config"]
