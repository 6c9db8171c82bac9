"""CUDA kernel layer (drop-in for mlx_gsq/runtime/kernels/__init__.py)."""
from .registry import DECODERS, SUPPORTED_QUANT_TYPES, decode, decode_weight
from .qmv import quantized_matvec
from .qmm import QMM_MIN_ROWS, quantized_matmul
from .embedding import iq2_s_embedding, packed_embedding

__all__ = ["DECODERS", "SUPPORTED_QUANT_TYPES", "decode", "decode_weight", "quantized_matvec",
           "quantized_matmul", "QMM_MIN_ROWS", "iq2_s_embedding", "packed_embedding"]
