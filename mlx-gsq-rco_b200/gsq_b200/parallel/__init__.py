"""Output-row tensor parallelism (NCCL all-gather over NVLink)."""
from .tp import RowParallelLinear, gather_rows, shard_bounds, shard_packed, shard_weight

__all__ = ["RowParallelLinear", "gather_rows", "shard_bounds", "shard_packed", "shard_weight"]
