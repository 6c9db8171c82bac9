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


class PackedModelStore:
    """Packed weights of an ``mlx-gsq-packed-v1`` safetensors container
    (``mlx_gsq/runtime/store.py:26-95``), loaded to the GPU.

    The container (written by ``gsq_b200.gguf.convert_gguf_to_safetensors``)
    holds each GGUF tensor's packed bytes as a one-dimensional U8 tensor; the
    quantization metadata comes from the sidecar manifest when present, else
    from the ``tensor_quantization`` JSON embedded in the safetensors metadata.
    ``weight(name)`` reads the tensor's byte range into pinned host memory and
    copies it to a CUDA uint8 tensor (``device=None`` keeps it on the host).
    """

    def __init__(self, model_path, manifest_path=None, device="cuda"):
        import json
        from pathlib import Path

        from ..gguf import CONTAINER_FORMAT, manifest_path_for, read_safetensors_header
        self.path = Path(model_path).expanduser().resolve()
        self.device = device
        header, self._data0 = read_safetensors_header(self.path)
        self.metadata = header.pop("__metadata__", {})
        if self.metadata.get("format") != CONTAINER_FORMAT:
            raise ValueError("safetensors metadata does not describe an mlx-gsq model")
        mfile = Path(manifest_path) if manifest_path else manifest_path_for(self.path)
        if mfile.exists():
            self.manifest = json.loads(mfile.read_text())
        else:
            embedded = json.loads(self.metadata["tensor_quantization"])
            self.manifest = {"format": CONTAINER_FORMAT, "tensors": {
                name: {"name": name, "gguf_shape": e["gguf_shape"], "logical_shape": e["logical_shape"],
                       "quantization_type": e["qtype"], "quantization_type_id": e["qtype_id"],
                       "num_elements": e["num_elements"], "num_bytes": int(header[name]["shape"][0])}
                for name, e in embedded.items()}}
        if self.manifest.get("format") != CONTAINER_FORMAT:
            raise ValueError("unsupported packed model format")
        if set(header) != set(self.manifest["tensors"]):
            raise ValueError("manifest and safetensors tensor names differ")
        for name, e in header.items():
            if e["dtype"] != "U8" or len(e["shape"]) != 1:
                raise ValueError(f"{name} is not a packed U8 tensor")
        self._entries = header

    def __len__(self) -> int:
        return len(self._entries)

    def __contains__(self, name: str) -> bool:
        return name in self._entries

    def names(self) -> list[str]:
        return list(self._entries)

    def weight(self, name: str, device="default") -> PackedWeight:
        from ..gguf import _to_device
        info = self.manifest["tensors"][name]
        lo, hi = self._entries[name]["data_offsets"]
        if hi - lo != info["num_bytes"]:
            raise ValueError(f"invalid packed data for {name}")
        data = _to_device(self.path, self._data0 + lo, hi - lo, self.device if device == "default" else device)
        return PackedWeight(name=name, data=data, gguf_shape=tuple(info["gguf_shape"]),
                            logical_shape=tuple(info["logical_shape"]), quantization_type=info["quantization_type"],
                            quantization_type_id=info["quantization_type_id"], num_elements=info["num_elements"],
                            num_bytes=info["num_bytes"])

    def materialize_plain(self, name: str) -> torch.Tensor:
        """An unquantized F32 / F16 / BF16 tensor in its own dtype and logical
        shape (no numeric conversion; ``store.py:88-95``)."""
        w = self.weight(name)
        dtypes = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16}
        if w.quantization_type not in dtypes:
            raise TypeError(f"{name} is {w.quantization_type}; a quantized kernel is required")
        return w.data.view(dtypes[w.quantization_type]).reshape(w.logical_shape)

    def model_weights(self) -> dict:
        """Every tensor by name, as ``gsq_b200.models.build_qwen35`` takes
        them: packed types as ``PackedWeight``, plain tensors as fp32."""
        from ..gguf import PACKED_IDS, plain_tensor
        out = {}
        for name in self._entries:
            w = self.weight(name)
            out[name] = w if w.quantization_type_id in PACKED_IDS else plain_tensor(w)
        return out
