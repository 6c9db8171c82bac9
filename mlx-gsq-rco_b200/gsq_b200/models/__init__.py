"""Model harness over the packed-weight kernels (mirrors mlx_gsq/models)."""
from .qwen35 import (Qwen35, Qwen35Config, build_qwen35, build_qwen35_head_split, default_type_mix,
                     head_split_weights, random_weights, tensor_shapes)

__all__ = ["Qwen35", "Qwen35Config", "build_qwen35", "build_qwen35_head_split", "default_type_mix",
           "head_split_weights", "random_weights", "tensor_shapes"]
