"""Output-row tensor parallelism: NCCL all-gather, or the gather fused into the matvec."""
from .gather import GatherRegion, quantized_matmul_gather, quantized_matvec_gather
from .tp import RowParallelLinear, gather_rows, shard_bounds, shard_packed, shard_weight

__all__ = ["GatherRegion", "RowParallelLinear", "gather_rows", "quantized_matmul_gather", "quantized_matvec_gather",
           "shard_bounds", "shard_packed", "shard_weight"]
