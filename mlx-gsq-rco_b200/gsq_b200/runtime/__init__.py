"""Runtime: packed weight container and the CUDA kernel layer."""
from .store import PackedWeight

__all__ = ["PackedWeight"]
