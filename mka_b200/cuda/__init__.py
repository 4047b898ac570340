"""Op API of the reference's mka.cuda package (mka/cuda/__init__.py, ops.py)."""
from ..ops import fastmka_attn, fused_route_mka_attn, has_fastmka_cuda, has_fused_route_mka_cuda

__all__ = ["fastmka_attn", "fused_route_mka_attn", "has_fastmka_cuda", "has_fused_route_mka_cuda"]
