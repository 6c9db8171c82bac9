"""gsq_b200: B200-native (sm_100a) packed-GGUF QMV / QMM / embedding gather.

Drop-in for the hot path of mlx-GSQ-RCO (``mlx_gsq.nn``, ``mlx_gsq.runtime.kernels``,
``mlx_gsq.quant`` block layouts).  Kernels live in ``gsq_b200/_lib/libgsq_b200.so``
(C ABI: include/gsq_b200.h); there is no CPU fallback.
"""
from .quant.layouts import QUANT_BLOCK_SIZES, SUPPORTED_QUANT_TYPES, GGMLQuantizationType
from .runtime.store import PackedWeight

__version__ = "0.1.0"
__all__ = ["QUANT_BLOCK_SIZES", "SUPPORTED_QUANT_TYPES", "GGMLQuantizationType", "PackedWeight", "__version__"]
