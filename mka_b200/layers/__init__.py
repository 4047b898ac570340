from .fastmka import FastMKAAttention, FastMKAConfig
from .session_memory import causal_prefix_ema, repeat_retrieval_to_length

__all__ = ["FastMKAAttention", "FastMKAConfig", "causal_prefix_ema", "repeat_retrieval_to_length"]
