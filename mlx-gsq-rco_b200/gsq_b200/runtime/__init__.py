"""Runtime: packed weight container and the CUDA kernel layer."""
from .store import PackedModelStore, PackedWeight

__all__ = ["PackedModelStore", "PackedWeight"]
