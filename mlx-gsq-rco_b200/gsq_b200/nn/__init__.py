"""GSQ-aware torch layers (drop-in for mlx_gsq/nn/__init__.py)."""
from .linear import GSQLinear
from .embedding import GSQEmbedding

__all__ = ["GSQLinear", "GSQEmbedding"]
