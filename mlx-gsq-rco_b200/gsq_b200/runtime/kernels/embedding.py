"""Packed embedding row lookup.

``iq2_s_embedding`` keeps the reference's name and contract
(``mlx_gsq/runtime/kernels/embedding.py:28-36``: ``ValueError`` unless
``dimensions % 256 == 0`` and the payload is ``vocab*(dim/256)*82`` bytes;
default dtype bf16).  ``packed_embedding`` is the same gather for any of the
eleven types (the reference handles IQ2_S only; the Qwen3.5 config uses
Q6_K embeddings).  Rows are decoded bit-exactly in fp32, then rounded once
to the output dtype.  The work runs in ``gsq_embed`` (csrc/dequant_embed.cu).
"""
from __future__ import annotations

import torch

from ... import _lib
from ...quant.layouts import QUANT_BLOCK_SIZES, SUPPORTED_QUANT_TYPES, type_id


def packed_embedding(ids: torch.Tensor, packed: torch.Tensor, *, qtype: str, vocab_size: int, dimensions: int,
                     dtype: torch.dtype | None = None) -> torch.Tensor:
    if qtype not in SUPPORTED_QUANT_TYPES:
        raise NotImplementedError(qtype)
    if dimensions % 256:
        raise ValueError("embedding dimensions must be divisible by 256")
    tid = type_id(qtype)
    expected = vocab_size * (dimensions // 256) * QUANT_BLOCK_SIZES[tid][1]
    if packed.numel() != expected:
        raise ValueError("packed embedding size mismatch")
    dev = _lib.require_cuda(ids, packed)
    dtype = dtype or torch.bfloat16
    flat = ids.reshape(-1).to(torch.int32).contiguous()
    out = torch.empty((flat.numel(), dimensions), dtype=dtype, device=dev)
    code = _lib.load().gsq_embed(tid, flat.data_ptr(), flat.numel(), packed.reshape(-1).contiguous().data_ptr(),
                                 vocab_size, dimensions, out.data_ptr(), _lib.DTYPE_CODES[dtype],
                                 _lib.stream_ptr(dev))
    _lib.check(code)
    return out.reshape(*ids.shape, dimensions)


def iq2_s_embedding(ids, packed, *, vocab_size: int, dimensions: int, dtype=None):
    if dimensions % 256:
        raise ValueError("embedding dimensions must be divisible by 256")
    if packed.numel() != vocab_size * (dimensions // 256) * 82:
        raise ValueError("packed embedding size mismatch")
    return packed_embedding(ids, packed, qtype="IQ2_S", vocab_size=vocab_size, dimensions=dimensions, dtype=dtype)
