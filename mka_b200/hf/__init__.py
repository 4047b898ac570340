from .attention import HFFastMKAAttention
from .cache import StaticKVCache
from .norm import FusedRMSNorm, apply_norm_fusion
from .patch import HFPatchConfig, apply_hf_attention_patch, parse_patch_config

__all__ = ["HFFastMKAAttention", "StaticKVCache", "FusedRMSNorm", "apply_norm_fusion", "HFPatchConfig",
           "apply_hf_attention_patch", "parse_patch_config"]
