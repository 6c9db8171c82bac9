"""Packed weight container.

``PackedWeight`` keeps the reference's frozen dataclass and field names
(``mlx_gsq/runtime/store.py:10-23``); ``data`` is a flat uint8 CUDA tensor of
the unmodified GGUF packed bytes.  ``PackedWeight.from_packed`` builds one
from a packed payload and its logical ``(out_features, in_features)`` shape.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from ..quant.layouts import QUANT_BLOCK_SIZES, type_id


@dataclass(frozen=True)
class PackedWeight:
    name: str
    data: Any
    gguf_shape: tuple[int, ...]
    logical_shape: tuple[int, ...]
    quantization_type: str
    quantization_type_id: int
    num_elements: int
    num_bytes: int

    @property
    def is_quantized(self) -> bool:
        return self.quantization_type not in {"F32", "F16", "BF16"}

    @classmethod
    def from_packed(cls, name: str, packed, qtype: str, logical_shape: tuple[int, ...],
                    device: torch.device | str | None = "cuda") -> "PackedWeight":
        tid = type_id(qtype)
        elems, bb = QUANT_BLOCK_SIZES[tid]
        numel = int(np.prod(logical_shape))
        if logical_shape[-1] % elems:
            raise ValueError(f"{name}: row width {logical_shape[-1]} is not a multiple of {elems}")
        nbytes = numel // elems * bb
        if isinstance(packed, np.ndarray):
            data = torch.from_numpy(np.ascontiguousarray(packed.reshape(-1)).view(np.uint8))
        else:
            data = packed.reshape(-1)
        if data.dtype != torch.uint8 or data.numel() != nbytes:
            raise ValueError(f"invalid packed data for {name}")
        if device is not None:
            data = data.to(device)
        return cls(name=name, data=data, gguf_shape=tuple(reversed(logical_shape)),
                   logical_shape=tuple(logical_shape), quantization_type=qtype, quantization_type_id=tid,
                   num_elements=numel, num_bytes=nbytes)
