"""Head-split layouts of the model's layers, and the packed-matrix selections
they need (host side).

Row-split tensor parallelism (``tp.py``, ``gather.py``) gives every rank a
slice of each projection's output rows. Every rank then needs the whole
output, so each projection ends in a gather, and the blocks between the
projections (gated-DeltaNet recurrence, attention) run on every rank. A
head-split layout keeps whole heads on a rank instead:

  * gated-DeltaNet (``mlx_gsq/models/qwen35.py:48-106``): a rank owns a run
    of key heads and every value head that reads one of them. Value head h
    reads key head ``h % nk`` (the cyclic routing of ``qwen35.py:87-94``).
    So with key heads ``[r*m, (r+1)*m)`` the rank's value heads are
    ``t*nk + r*m + i`` for repeat t and i < m. In that order, local value
    head j reads local key head ``j % m``, the same cyclic rule with nk = m,
    so the block's kernel runs unchanged on the local heads;
  * gated GQA attention: a rank owns a run of query heads and the key/value
    heads they read (query head h reads key/value head ``h // (nq/nkv)``).
    When a rank has fewer query heads than a group, the ranks of one group
    share that group's key/value head;
  * SwiGLU FFN: a rank owns a run of 256-wide blocks of the intermediate
    width: those rows of gate and up, the same input blocks of down.

The projection that reads a block's local heads (``ssm_out``,
``attn_output``, ``ffn_down``) then holds only the input blocks of those
heads. Each rank computes a partial output of full width, and the ranks sum
the partials (one reduce per block instead of one gather per projection;
``InputParallelLinear`` in ``tp.py``).

Both selections are byte rearrangements of a packed matrix, with no
re-quantisation. Row n of an N x K matrix is the contiguous span
``[n*rb, (n+1)*rb)``, and input block j of that row is bytes
``[j*bb, (j+1)*bb)`` of the span (``rb = (K/256)*bb``, ``bb`` the block's
bytes). A head's input columns must therefore cover whole 256-wide blocks;
the plans check that.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

from ..quant.layouts import QUANT_BLOCK_SIZES, type_id

QK = 256  # inputs per packed block


def _check_rank(world: int, rank: int) -> None:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of {world}")


def _blocks_of_columns(cols: Sequence[int], what: str) -> list[int]:
    """The 256-wide input blocks that exactly cover the sorted column runs
    ``cols`` (a flat list of column indices)."""
    if len(cols) % QK:
        raise ValueError(f"{what}: {len(cols)} columns are not whole 256-wide blocks")
    blocks = []
    for i in range(0, len(cols), QK):
        c0 = cols[i]
        if c0 % QK or list(cols[i:i + QK]) != list(range(c0, c0 + QK)):
            raise ValueError(f"{what}: columns {c0}.. do not fill one aligned 256-wide block")
        blocks.append(c0 // QK)
    return blocks


@dataclass(frozen=True)
class LinearAttentionHeads:
    """One rank's heads of a gated-DeltaNet layer (global indices, local order)."""
    nk: int
    nv: int
    key_heads: tuple[int, ...]
    value_heads: tuple[int, ...]

    def qkv_rows(self, dk: int, dv: int) -> list[int]:
        """Rows of the q|k|v projection (``attn_qkv``: nk*dk query rows, nk*dk
        key rows, nv*dv value rows), also the depthwise conv channels, in the
        local layout q | k | v that the block's kernel takes."""
        q = [h * dk + i for h in self.key_heads for i in range(dk)]
        k = [self.nk * dk + h * dk + i for h in self.key_heads for i in range(dk)]
        v = [2 * self.nk * dk + h * dv + i for h in self.value_heads for i in range(dv)]
        return q + k + v

    def gate_rows(self, dv: int) -> list[int]:
        """Rows of the output gate z (``attn_gate``, nv*dv rows)."""
        return [h * dv + i for h in self.value_heads for i in range(dv)]

    def out_blocks(self, dv: int) -> list[int]:
        """Input blocks of the output projection (``ssm_out``, nv*dv inputs)
        that the local value heads' outputs feed, in the local order."""
        return _blocks_of_columns([h * dv + i for h in self.value_heads for i in range(dv)], "ssm_out")


def linear_attention_heads(nk: int, nv: int, world: int, rank: int, dv: int = 128) -> LinearAttentionHeads:
    """Key heads ``[r*m, (r+1)*m)`` (m = nk/world) and the value heads that
    read them, ordered so that local value head j reads local key head
    ``j % m``. The local value heads must fill whole 256-wide input blocks
    of the output projection (128-wide heads: an even number of key heads
    per rank)."""
    _check_rank(world, rank)
    if nk <= 0 or nv % nk:
        raise ValueError("value heads must be a multiple of key heads")
    if nk % world:
        raise ValueError(f"{nk} key heads do not split over {world} ranks")
    m = nk // world
    keys = tuple(range(rank * m, (rank + 1) * m))
    values = tuple(t * nk + k for t in range(nv // nk) for k in keys)
    plan = LinearAttentionHeads(nk, nv, keys, values)
    plan.out_blocks(dv)  # raises unless the local value heads fill whole blocks
    return plan


@dataclass(frozen=True)
class AttentionHeads:
    """One rank's heads of a gated GQA attention layer (global indices)."""
    nq: int
    nkv: int
    query_heads: tuple[int, ...]
    kv_heads: tuple[int, ...]

    def q_rows(self, hd: int) -> list[int]:
        """Rows of ``attn_q`` (per query head hd query rows then hd gate rows)."""
        return [h * 2 * hd + i for h in self.query_heads for i in range(2 * hd)]

    def kv_rows(self, hd: int) -> list[int]:
        """Rows of ``attn_k`` and of ``attn_v`` (hd rows per key/value head)."""
        return [h * hd + i for h in self.kv_heads for i in range(hd)]

    def out_blocks(self, hd: int) -> list[int]:
        """Input blocks of ``attn_output`` fed by the local query heads."""
        return _blocks_of_columns([h * hd + i for h in self.query_heads for i in range(hd)], "attn_output")


def attention_heads(nq: int, nkv: int, world: int, rank: int, hd: int = 256) -> AttentionHeads:
    """Query heads ``[r*m, (r+1)*m)`` (m = nq/world) and the key/value heads
    they read. Local query head j reads local key/value head
    ``j // (m / len(kv_heads))``: the grouped rule of the whole layer."""
    _check_rank(world, rank)
    if nkv <= 0 or nq % nkv:
        raise ValueError("query heads must be a multiple of key/value heads")
    if nq % world:
        raise ValueError(f"{nq} query heads do not split over {world} ranks")
    g, m = nq // nkv, nq // world
    if m % g and g % m:
        raise ValueError(f"{m} query heads per rank do not align with groups of {g}")
    queries = tuple(range(rank * m, (rank + 1) * m))
    kvs = tuple(sorted({h // g for h in queries}))
    plan = AttentionHeads(nq, nkv, queries, kvs)
    plan.out_blocks(hd)
    return plan


def ffn_blocks(intermediate: int, world: int, rank: int) -> range:
    """256-wide blocks of the FFN's intermediate width owned by ``rank``: as
    even as whole blocks allow (the first ``blocks % world`` ranks hold one
    more). Gate and up keep rows ``[256*b0, 256*b1)``, down the same input
    blocks."""
    _check_rank(world, rank)
    if intermediate <= 0 or intermediate % QK:
        raise ValueError("the intermediate width must be a positive multiple of 256")
    kb = intermediate // QK
    if kb < world:
        raise ValueError(f"{kb} blocks cannot give each of {world} ranks one")
    per, extra = divmod(kb, world)
    b0 = rank * per + min(rank, extra)
    return range(b0, b0 + per + (1 if rank < extra else 0))


def _as_blocks(packed: torch.Tensor, qtype: str, out_features: int, in_features: int) -> torch.Tensor:
    elems, bb = QUANT_BLOCK_SIZES[type_id(qtype)]
    if elems != QK or in_features % QK:
        raise ValueError("packed rows must be whole 256-wide blocks")
    flat = packed.reshape(-1)
    kb = in_features // QK
    if flat.numel() != out_features * kb * bb:
        raise ValueError("packed size does not match the matrix shape")
    return flat.view(out_features, kb, bb)


def take_rows(packed: torch.Tensor, qtype: str, out_features: int, in_features: int,
              rows: Sequence[int]) -> torch.Tensor:
    """The packed matrix of the given output rows, in the given order (a copy
    on the same device, flat uint8)."""
    m = _as_blocks(packed, qtype, out_features, in_features)
    idx = torch.as_tensor(list(rows), dtype=torch.long, device=m.device)
    if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= out_features):
        raise ValueError("row index outside the matrix")
    return m.index_select(0, idx).reshape(-1).contiguous()


def take_input_blocks(packed: torch.Tensor, qtype: str, out_features: int, in_features: int,
                      blocks: Sequence[int]) -> torch.Tensor:
    """The packed matrix restricted to the given 256-wide input blocks, in the
    given order: an out_features x (256*len(blocks)) packed matrix (a copy
    on the same device, flat uint8). Its product with the matching columns
    of x is this rank's partial of the full product."""
    m = _as_blocks(packed, qtype, out_features, in_features)
    idx = torch.as_tensor(list(blocks), dtype=torch.long, device=m.device)
    if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= m.shape[1]):
        raise ValueError("input block outside the matrix")
    return m.index_select(1, idx).reshape(-1).contiguous()
