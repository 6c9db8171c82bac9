"""Tensor parallelism of packed projections: output-row splits (NCCL all-gather,
or the gather fused into the matvec / matmul), input-block splits with a sum
reduction, and the head-split layer layouts that use them."""
from .gather import GatherRegion, quantized_matmul_gather, quantized_matvec_gather
from .heads import (AttentionHeads, LinearAttentionHeads, attention_heads, ffn_blocks, linear_attention_heads,
                    take_input_blocks, take_rows)
from .tp import (InputParallelLinear, RowParallelLinear, block_bounds, gather_rows, reduce_partials, shard_bounds,
                 shard_packed, shard_weight)

__all__ = ["AttentionHeads", "GatherRegion", "InputParallelLinear", "LinearAttentionHeads", "RowParallelLinear",
           "attention_heads", "block_bounds", "ffn_blocks", "gather_rows", "linear_attention_heads",
           "quantized_matmul_gather", "quantized_matvec_gather", "reduce_partials", "shard_bounds", "shard_packed",
           "shard_weight", "take_input_blocks", "take_rows"]
