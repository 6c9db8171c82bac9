"""Decode registry: dispatch by quant-type name to the bit-exact CUDA decoder.

Mirrors ``mlx_gsq/runtime/kernels/registry.py:8-46`` (``SUPPORTED_QUANT_TYPES``,
``DECODERS``, ``decode``, ``decode_weight``): same names, same argument
meaning, same errors (``NotImplementedError`` for an unknown type in
``decode``, ``TypeError`` for a non-quantized weight in ``decode_weight``).
Output is a flat float32 CUDA tensor, bit-identical to gguf-py.
"""
from __future__ import annotations

import torch

from ... import _lib
from ...quant.layouts import QUANT_BLOCK_SIZES, SUPPORTED_QUANT_TYPES, type_id


def _decoder(qtype: str):
    tid = type_id(qtype)
    bb = QUANT_BLOCK_SIZES[tid][1]

    def decode_fn(packed: torch.Tensor) -> torch.Tensor:
        dev = _lib.require_cuda(packed)
        if packed.dtype != torch.uint8:
            raise TypeError("packed input must be uint8")
        flat = packed.reshape(-1)
        if not flat.is_contiguous():
            flat = flat.contiguous()
        if flat.numel() % bb:
            raise ValueError(f"{qtype} payload is not block aligned")
        nblocks = flat.numel() // bb
        out = torch.empty(nblocks * 256, dtype=torch.float32, device=dev)
        _lib.check(_lib.load().gsq_dequant(tid, flat.data_ptr(), nblocks, out.data_ptr(), _lib.stream_ptr(dev)))
        return out

    decode_fn.__name__ = f"decode_{qtype.lower()}"
    return decode_fn


DECODERS = {q: _decoder(q) for q in SUPPORTED_QUANT_TYPES}


def decode(packed: torch.Tensor, qtype: str) -> torch.Tensor:
    try:
        decoder = DECODERS[qtype]
    except KeyError as error:
        raise NotImplementedError(f"validated CUDA decoder not available for {qtype}") from error
    return decoder(packed)


def decode_weight(weight, *, block_count: int | None = None) -> torch.Tensor:
    """Route a PackedWeight to its decoder using its embedded metadata."""
    qtype = weight.quantization_type
    if qtype not in SUPPORTED_QUANT_TYPES:
        raise TypeError(f"{weight.name} is not a supported quantized weight: {qtype}")
    data = weight.data
    if block_count is not None:
        block_bytes = QUANT_BLOCK_SIZES[weight.quantization_type_id][1]
        data = data[: block_count * block_bytes]
    return decode(data, qtype)
