"""Packed mixed-quant linear layer.

Same constructor and call contract as ``mlx_gsq/nn/linear.py:6-24``:
``GSQLinear(weight, bias=None)`` reads ``weight.data``, ``logical_shape`` and
``quantization_type``; ``__call__(x)`` computes ``rows = x.numel() //
in_features`` and runs the fused matvec for one row, the tiled matmul
otherwise, then adds the bias.
"""
from __future__ import annotations

import torch

from ..runtime.kernels.qmm import quantized_matmul
from ..runtime.kernels.qmv import quantized_matvec


class GSQLinear(torch.nn.Module):
    def __init__(self, weight, bias=None):
        super().__init__()
        self.packed_weight = weight.data
        self.bias = bias
        self.in_features = weight.logical_shape[1]
        self.out_features = weight.logical_shape[0]
        self.qtype = weight.quantization_type

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        rows = x.numel() // self.in_features
        kw = dict(qtype=self.qtype, out_features=self.out_features, in_features=self.in_features,
                  out_dtype=out_dtype)
        if rows == 1:
            y = quantized_matvec(x, self.packed_weight, **kw)
        else:
            y = quantized_matmul(x, self.packed_weight, **kw)
        return y if self.bias is None else y + self.bias

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, qtype={self.qtype}"
