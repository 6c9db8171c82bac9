"""Packed embedding layer.

Same constructor and call contract as ``mlx_gsq/nn/embedding.py:4-11``
(``GSQEmbedding(weight, dtype=None)``, ``__call__(ids)``), extended from IQ2_S
to all eleven packed types.
"""
from __future__ import annotations

import torch

from ..quant.layouts import SUPPORTED_QUANT_TYPES
from ..runtime.kernels.embedding import packed_embedding


class GSQEmbedding(torch.nn.Module):
    def __init__(self, weight, dtype=None):
        super().__init__()
        if weight.quantization_type not in SUPPORTED_QUANT_TYPES:
            raise NotImplementedError(weight.quantization_type)
        self.packed_weight = weight.data
        self.qtype = weight.quantization_type
        self.num_embeddings = weight.logical_shape[0]
        self.dimensions = weight.logical_shape[1]
        self.dtype = dtype

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        return packed_embedding(ids, self.packed_weight, qtype=self.qtype, vocab_size=self.num_embeddings,
                                dimensions=self.dimensions, dtype=self.dtype)
