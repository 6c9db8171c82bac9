"""Block layouts, codebooks and synthetic packed data."""
from .layouts import (GGMLQuantizationType, LAYOUTS, QUANT_BLOCK_SIZES, SUPPORTED_QUANT_TYPES, block_bytes,
                      packed_bytes, type_id)

__all__ = ["GGMLQuantizationType", "LAYOUTS", "QUANT_BLOCK_SIZES", "SUPPORTED_QUANT_TYPES", "block_bytes",
           "packed_bytes", "type_id"]
