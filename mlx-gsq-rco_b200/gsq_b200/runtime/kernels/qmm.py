"""Tiled dequantize + matmul on tcgen05 tensor cores (prefill path).

Mirrors ``mlx_gsq/runtime/kernels/qmm.py:559-594`` (``quantized_matmul``):
same keyword arguments (``kt`` is accepted for signature compatibility; the
B200 kernel's K tiling is fixed by its pipeline), same validation, output
``x.shape[:-1] + (out_features,)`` in ``x.dtype`` unless ``out_dtype`` is
given.  Accumulation is fp32 in TMEM; weights are decoded to fp16 tiles.
The work runs in ``gsq_qmm`` (csrc/qmm.cu).
"""
from __future__ import annotations

import torch

from ... import _lib
from ...quant.layouts import QUANT_BLOCK_SIZES, SUPPORTED_QUANT_TYPES, GGMLQuantizationType

QMM_MIN_ROWS = 8  # qmm.py:26


def quantized_matmul(x: torch.Tensor, packed: torch.Tensor, *, qtype: str, out_features: int, in_features: int,
                     kt: int = 256, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    if qtype not in SUPPORTED_QUANT_TYPES:
        raise NotImplementedError(f"no tiled QMM kernel for {qtype}")
    if kt not in (128, 256):
        raise ValueError(f"unsupported kt {kt}")
    type_id = int(GGMLQuantizationType[qtype])
    block_elements, block_bytes = QUANT_BLOCK_SIZES[type_id]
    if block_elements != 256 or in_features % 256:
        raise ValueError(f"invalid {qtype} matrix width")
    expected = out_features * (in_features // 256) * block_bytes
    if packed.numel() != expected:
        raise ValueError(f"packed size {packed.numel()} != expected {expected}")
    if x.shape[-1] != in_features:
        raise ValueError("input feature size mismatch")
    if x.dtype not in _lib.DTYPE_CODES:
        raise TypeError(f"unsupported activation dtype {x.dtype}")
    dev = _lib.require_cuda(x, packed)
    original = x.shape[:-1]
    rows = x.numel() // in_features
    flat = x.reshape(rows, in_features).contiguous()
    if flat.data_ptr() % 16:
        flat = flat.clone()  # TMA / vector loads need 16-byte alignment
    pk = packed.reshape(-1).contiguous()
    out_dtype = out_dtype or x.dtype
    if out_dtype not in _lib.DTYPE_CODES:
        raise TypeError(f"unsupported output dtype {out_dtype}")
    y = torch.empty((rows, out_features), dtype=out_dtype, device=dev)  # rounded once from the fp32 sums
    lib = _lib.load()
    xcode = _lib.DTYPE_CODES[flat.dtype]
    need = lib.gsq_qmm_workspace_size(type_id, out_features, in_features, rows, xcode)
    ws = _lib.workspaces.get(dev, need, "qmm")
    code = lib.gsq_qmm(type_id, flat.data_ptr(), xcode, pk.data_ptr(), out_features, in_features, rows,
                       y.data_ptr(), _lib.DTYPE_CODES[out_dtype], ws.data_ptr() if ws is not None else None,
                       ws.numel() if ws is not None else 0, _lib.stream_ptr(dev))
    _lib.check(code)
    return y.reshape(*original, out_features)
