"""Fused dequantize + matvec (decode path).

Mirrors ``mlx_gsq/runtime/kernels/qmv.py:537-576`` (``quantized_matvec``):
same keyword arguments, same validation (``ValueError`` for a bad width,
payload size or feature size; ``NotImplementedError`` for an unknown type),
same reroute of inputs with ``rows >= QMM_MIN_ROWS`` to the tiled QMM
(``qmv.py:548-549``), output shaped ``x.shape[:-1] + (out_features,)`` in
``x.dtype`` (``qmv.py:557-575``) unless ``out_dtype`` says otherwise.
The work runs in ``gsq_qmv`` (csrc/qmv.cu).
"""
from __future__ import annotations

import torch

from ... import _lib
from ...quant.layouts import QUANT_BLOCK_SIZES, GGMLQuantizationType
from .qmm import QMM_MIN_ROWS, quantized_matmul


# gsq_qmv_workspace_size per (type id, N, K, rows): a pure function of the shape.
_WORKSPACE_BYTES: dict[tuple[int, int, int, int], int] = {}


def _validate(x, packed, qtype, out_features, in_features):
    try:
        type_id = int(GGMLQuantizationType[qtype])
    except KeyError as error:
        raise NotImplementedError(f"no packed kernel for {qtype}") from error
    block_elements, block_bytes = QUANT_BLOCK_SIZES[type_id]
    if block_elements != 256 or in_features % 256:
        raise ValueError(f"invalid {qtype} matrix width")
    expected = out_features * (in_features // 256) * block_bytes
    if packed.numel() != expected:
        raise ValueError(f"packed size {packed.numel()} != expected {expected}")
    if x.shape[-1] != in_features:
        raise ValueError("input feature size mismatch")
    if packed.dtype != torch.uint8:
        raise TypeError("packed weights must be uint8")
    if x.dtype not in _lib.DTYPE_CODES:
        raise TypeError(f"unsupported activation dtype {x.dtype}")
    return type_id


def quantized_matvec(x: torch.Tensor, packed: torch.Tensor, *, qtype: str, out_features: int, in_features: int,
                     out_dtype: torch.dtype | None = None) -> torch.Tensor:
    type_id = _validate(x, packed, qtype, out_features, in_features)
    dev = _lib.require_cuda(x, packed)
    original = x.shape[:-1]
    rows = x.numel() // in_features
    flat = x.reshape(rows, in_features)
    if rows >= QMM_MIN_ROWS:
        return quantized_matmul(flat, packed, qtype=qtype, out_features=out_features, in_features=in_features,
                                out_dtype=out_dtype).reshape(*original, out_features)
    out_dtype = out_dtype or x.dtype
    flat = flat.contiguous()
    if flat.data_ptr() % 16:
        flat = flat.clone()  # the kernel reads activations with 16-byte loads
    pk = packed.reshape(-1).contiguous()
    y = torch.empty((rows, out_features), dtype=out_dtype, device=dev)
    lib = _lib.load()
    key = (type_id, out_features, in_features, rows)
    need = _WORKSPACE_BYTES.get(key)
    if need is None:
        need = _WORKSPACE_BYTES[key] = lib.gsq_qmv_workspace_size(type_id, out_features, in_features, rows)
    ws = _lib.workspaces.get(dev, need, "qmv")
    code = lib.gsq_qmv(type_id, flat.data_ptr(), _lib.DTYPE_CODES[flat.dtype], pk.data_ptr(), out_features,
                       in_features, rows, y.data_ptr(), _lib.DTYPE_CODES[out_dtype],
                       ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                       _lib.stream_ptr(dev))
    _lib.check(code)
    return y.reshape(*original, out_features)
