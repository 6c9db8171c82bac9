"""Output-row tensor parallelism for packed projections.

The reference has no parallelism of its own (its only trace is mlx-lm's
unexercised ``all_sum`` hook, ``mlx_gsq/models/qwen35.py:104-105``).  Row n of
a packed matrix is one contiguous byte span ``[n*rb, (n+1)*rb)`` with
``rb = (K/256)*block_bytes``, so a projection shards across ranks by output
rows with no repacking: rank r of P keeps rows ``[r*N/P, (r+1)*N/P)`` and
computes its slice of y with the local QMV/QMM kernel; the slices are joined
with one NCCL ``all_gather_into_tensor`` over NVLink.

A projection can also split by 256-wide input blocks (``InputParallelLinear``):
each rank multiplies its blocks of every row with its part of x, and the
partial outputs are summed over the ranks.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..quant.layouts import QUANT_BLOCK_SIZES, type_id
from ..runtime.store import PackedWeight
from .heads import ffn_blocks, take_input_blocks


def shard_bounds(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) owned by ``rank``; requires n_rows % world == 0."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("invalid rank/world")
    if n_rows % world:
        raise ValueError(f"{n_rows} output rows do not split evenly over {world} ranks")
    per = n_rows // world
    return rank * per, (rank + 1) * per


def row_bytes(qtype: str, in_features: int) -> int:
    elems, bb = QUANT_BLOCK_SIZES[type_id(qtype)]
    return in_features // elems * bb


def shard_packed(packed: torch.Tensor, qtype: str, out_features: int, in_features: int, world: int,
                 rank: int) -> torch.Tensor:
    """Byte slice of the packed matrix holding this rank's output rows (a copy)."""
    lo, hi = shard_bounds(out_features, world, rank)
    rb = row_bytes(qtype, in_features)
    flat = packed.reshape(-1)
    if flat.numel() != out_features * rb:
        raise ValueError("packed size does not match the matrix shape")
    return flat[lo * rb:hi * rb].clone()


def shard_weight(weight: PackedWeight, world: int, rank: int) -> PackedWeight:
    n, k = weight.logical_shape
    data = shard_packed(weight.data, weight.quantization_type, n, k, world, rank)
    lo, hi = shard_bounds(n, world, rank)
    return PackedWeight(name=f"{weight.name}[rows {lo}:{hi}]", data=data, gguf_shape=(k, hi - lo),
                        logical_shape=(hi - lo, k), quantization_type=weight.quantization_type,
                        quantization_type_id=weight.quantization_type_id, num_elements=(hi - lo) * k,
                        num_bytes=data.numel())


def gather_rows(y_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-rank output slices (..., N/P) into (..., N), rank-major."""
    world = dist.get_world_size(group)
    if world == 1:
        return y_local
    lead = y_local.shape[:-1]
    cols = y_local.shape[-1]
    flat = y_local.reshape(-1, cols).contiguous()
    rows = flat.shape[0]
    out = torch.empty((world, rows, cols), dtype=flat.dtype, device=flat.device)
    if flat.device.type == "cuda":
        dist.all_gather_into_tensor(out, flat, group=group)
    else:
        parts = list(out.unbind(0))
        dist.all_gather(parts, flat, group=group)
        out = torch.stack(parts, 0)
    return out.permute(1, 0, 2).reshape(*lead, world * cols)


class RowParallelLinear(torch.nn.Module):
    """A packed projection split by output rows across the ranks of ``group``.

    ``forward(x)`` runs the local shard with the fused kernels (GSQLinear
    dispatch: matvec for few rows, tiled matmul otherwise) and joins the
    output slices, so every rank returns the full ``(..., out_features)``.
    Decode-sized inputs on CUDA (``fused_gather``) use the matvec with the
    gather fused in (one kernel, NVLink stores into every rank's copy, see
    ``gather.py``); other inputs use an NCCL all-gather after the kernel.
    """

    def __init__(self, weight: PackedWeight, group=None, bias: torch.Tensor | None = None, local_fn=None,
                 fused_gather: bool = True):
        super().__init__()
        from ..nn.linear import GSQLinear
        self.group = group
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world, self.rank = world, rank
        self.out_features, self.in_features = weight.logical_shape
        self.shard = shard_weight(weight, world, rank) if world > 1 else weight
        self.row0 = shard_bounds(self.out_features, world, rank)[0] if world > 1 else 0
        self.bias = bias
        self.local = local_fn or GSQLinear(self.shard)
        self.fused_gather = fused_gather and local_fn is None and 2 <= world <= 8
        self._regions: dict[int, object] = {}

    def _gathered_matvec(self, x: torch.Tensor) -> torch.Tensor:
        from .gather import GatherRegion, quantized_matvec_gather
        rows = x.numel() // self.in_features
        region = self._regions.get(rows)
        if region is None:
            region = self._regions[rows] = GatherRegion(rows, self.out_features, self.group, x.device)
        y = quantized_matvec_gather(x, self.shard.data, qtype=self.shard.quantization_type,
                                    out_features=self.out_features // self.world, in_features=self.in_features,
                                    region=region, row0=self.row0)
        y = y.reshape(*x.shape[:-1], self.out_features)
        return y if x.dtype == torch.float32 else y.to(x.dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from ..runtime.kernels.qmv import QMM_MIN_ROWS
        if self.world > 1 and self.fused_gather and x.is_cuda and x.numel() // self.in_features < QMM_MIN_ROWS:
            y = self._gathered_matvec(x)
        else:
            y = gather_rows(self.local(x), self.group) if self.world > 1 else self.local(x)
        return y if self.bias is None else y + self.bias

    def close(self) -> None:
        """Release the gather regions (collective: every rank calls it)."""
        for r in self._regions.values():
            r.close()
        self._regions.clear()


def block_bounds(in_features: int, world: int, rank: int) -> tuple[int, int]:
    """256-wide input blocks [b0, b1) owned by ``rank``: as even as whole
    blocks allow (the first ``blocks % world`` ranks hold one more)."""
    r = ffn_blocks(in_features, world, rank)
    return r.start, r.stop


def reduce_partials(y: torch.Tensor, group=None) -> torch.Tensor:
    """Sums the ranks' partial outputs in place (NCCL on CUDA tensors, the
    group's backend otherwise); every rank returns the same sum."""
    if dist.get_world_size(group) > 1:
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y


class InputParallelLinear(torch.nn.Module):
    """A packed projection split by 256-wide input blocks across the ranks
    of ``group``: the counterpart of ``RowParallelLinear`` for the
    projection that reads a head-split block's local outputs (``heads.py``).

    Rank r keeps every output row's input blocks ``blocks`` (by default an
    even run, ``block_bounds``; a head plan's ``out_blocks`` otherwise) and
    ``forward(x_local)`` multiplies them with its own inputs x_local (the
    matching columns of the full input, ``local_columns``), in fp32, then
    sums the partials over the ranks. Every rank returns the full
    ``(..., out_features)`` output, in x_local's dtype unless ``out_dtype``
    says otherwise."""

    def __init__(self, weight: PackedWeight, group=None, blocks=None, bias: torch.Tensor | None = None,
                 local_fn=None):
        super().__init__()
        from ..nn.linear import GSQLinear
        self.group = group
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world, self.rank = world, rank
        self.out_features, self.in_features = weight.logical_shape
        if blocks is None:
            blocks = range(*block_bounds(self.in_features, world, rank))
        self.blocks = tuple(int(b) for b in blocks)
        if not self.blocks:
            raise ValueError("a rank needs at least one input block")
        k_local = len(self.blocks) * 256
        data = take_input_blocks(weight.data, weight.quantization_type, self.out_features, self.in_features,
                                 self.blocks)
        self.shard = PackedWeight(name=f"{weight.name}[{len(self.blocks)} input blocks]", data=data,
                                  gguf_shape=(k_local, self.out_features),
                                  logical_shape=(self.out_features, k_local),
                                  quantization_type=weight.quantization_type,
                                  quantization_type_id=weight.quantization_type_id,
                                  num_elements=self.out_features * k_local, num_bytes=data.numel())
        self.bias = bias
        self.local = local_fn or GSQLinear(self.shard)
        self._local_fn = local_fn is not None
        self._columns: dict = {}  # column index tensor per device (local_columns)

    def local_columns(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's inputs: the columns of the full input x that its blocks read."""
        idx = self._columns.get(x.device)
        if idx is None:
            idx = self._columns[x.device] = torch.tensor([b * 256 + i for b in self.blocks for i in range(256)],
                                                         device=x.device)
        return x.index_select(-1, idx)

    def forward(self, x_local: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        if x_local.shape[-1] != len(self.blocks) * 256:
            raise ValueError("x_local must hold this rank's input columns")
        y = self.local(x_local) if self._local_fn else self.local(x_local, out_dtype=torch.float32)
        y = reduce_partials(y.float().contiguous(), self.group)
        if self.bias is not None:
            y = y + self.bias
        return y.to(out_dtype or x_local.dtype)
