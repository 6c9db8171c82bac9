"""GGUF quant type ids, block sizes and the 256-weight super-block layouts.

The type ids and the (elements, bytes) table are the GGML type traits that the
reference carries in ``mlx_gsq/gguf/parser.py:26-42`` (``GGMLQuantizationType``,
``QUANT_BLOCK_SIZES``). They are a file-format contract, so the values are the
same; the layout descriptions below are the byte offsets that the reference's
decoders read (``mlx_gsq/runtime/kernels/k_decode.py:17-81``,
``iq_lookup_decode.py:6-37``, ``iq3_s_decode.py:16-40``) and that gguf-py 0.19.0
``gguf/quants.py`` dequantizes.
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum


class GGMLQuantizationType(IntEnum):
    """GGML tensor type ids (``mlx_gsq/gguf/parser.py:26-32``)."""
    F32 = 0; F16 = 1; Q4_0 = 2; Q4_1 = 3; Q5_0 = 6; Q5_1 = 7; Q8_0 = 8; Q8_1 = 9
    Q2_K = 10; Q3_K = 11; Q4_K = 12; Q5_K = 13; Q6_K = 14; Q8_K = 15
    IQ2_XXS = 16; IQ2_XS = 17; IQ3_XXS = 18; IQ1_S = 19; IQ4_NL = 20
    IQ3_S = 21; IQ2_S = 22; IQ4_XS = 23; I8 = 24; I16 = 25; I32 = 26; I64 = 27
    F64 = 28; IQ1_M = 29; BF16 = 30; TQ1_0 = 34; TQ2_0 = 35; MXFP4 = 39; NVFP4 = 40


# (logical elements per block, stored bytes per block); ``parser.py:35-42``.
QUANT_BLOCK_SIZES: dict[int, tuple[int, int]] = {
    0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24),
    8: (32, 34), 9: (32, 36), 10: (256, 84), 11: (256, 110), 12: (256, 144),
    13: (256, 176), 14: (256, 210), 15: (256, 292), 16: (256, 66), 17: (256, 74),
    18: (256, 98), 19: (256, 50), 20: (32, 18), 21: (256, 110), 22: (256, 82),
    23: (256, 136), 24: (1, 1), 25: (1, 2), 26: (1, 4), 27: (1, 8), 28: (1, 8),
    29: (256, 56), 30: (1, 2), 34: (256, 54), 35: (256, 66), 39: (32, 17), 40: (64, 36),
}

# The eleven packed types the hot path supports (``registry.py:8-11``).
SUPPORTED_QUANT_TYPES: tuple[str, ...] = (
    "IQ1_M", "IQ1_S", "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS",
    "IQ3_S", "IQ4_XS", "Q2_K", "Q4_K", "Q6_K",
)

QK_K = 256


@dataclass(frozen=True)
class BlockLayout:
    """One 256-weight super-block: byte size and a field map for documentation."""
    name: str
    type_id: int
    block_bytes: int
    fields: tuple[tuple[str, int, int], ...]  # (field, byte offset, byte length)
    scale_unit: int  # weights sharing one sub-block scale

    @property
    def bits_per_weight(self) -> float:
        return self.block_bytes * 8 / QK_K


def _L(name, fields, unit):
    tid = int(GGMLQuantizationType[name])
    return BlockLayout(name, tid, QUANT_BLOCK_SIZES[tid][1], fields, unit)


# Field maps follow gguf-py 0.19.0 ``quants.py`` dequantize_blocks splits.
LAYOUTS: dict[str, BlockLayout] = {
    l.name: l for l in (
        _L("Q2_K", (("scales", 0, 16), ("qs", 16, 64), ("d", 80, 2), ("dmin", 82, 2)), 16),
        _L("Q4_K", (("d", 0, 2), ("dmin", 2, 2), ("scales", 4, 12), ("qs", 16, 128)), 32),
        _L("Q6_K", (("ql", 0, 128), ("qh", 128, 64), ("scales", 192, 16), ("d", 208, 2)), 16),
        _L("IQ4_XS", (("d", 0, 2), ("scales_h", 2, 2), ("scales_l", 4, 4), ("qs", 8, 128)), 32),
        _L("IQ2_XXS", (("d", 0, 2), ("qs", 2, 64)), 32),
        _L("IQ2_XS", (("d", 0, 2), ("qs", 2, 64), ("scales", 66, 8)), 16),
        _L("IQ2_S", (("d", 0, 2), ("qs", 2, 32), ("signs", 34, 32), ("qh", 66, 8), ("scales", 74, 8)), 16),
        _L("IQ3_XXS", (("d", 0, 2), ("qs", 2, 64), ("scales", 66, 32)), 32),
        _L("IQ3_S", (("d", 0, 2), ("qs", 2, 64), ("qh", 66, 8), ("signs", 74, 32), ("scales", 106, 4)), 32),
        _L("IQ1_S", (("d", 0, 2), ("qs", 2, 32), ("qh", 34, 16)), 32),
        _L("IQ1_M", (("qs", 0, 32), ("qh", 32, 16), ("scales", 48, 8)), 16),
    )
}

# Offsets of the fp16 super-block scale(s) in each layout.  IQ1_M has no
# contiguous fp16 field: its d is spread over the top nibbles of the four
# u16 scale words (gguf-py quants.py:1304-1308).
SCALE_FIELDS: dict[str, tuple[int, ...]] = {
    "Q2_K": (80, 82), "Q4_K": (0, 2), "Q6_K": (208,), "IQ4_XS": (0,),
    "IQ2_XXS": (0,), "IQ2_XS": (0,), "IQ2_S": (0,), "IQ3_XXS": (0,),
    "IQ3_S": (0,), "IQ1_S": (0,), "IQ1_M": (),
}


def type_id(qtype: str) -> int:
    return int(GGMLQuantizationType[qtype])


def block_bytes(qtype: str) -> int:
    return QUANT_BLOCK_SIZES[type_id(qtype)][1]


def packed_bytes(qtype: str, out_features: int, in_features: int) -> int:
    """Bytes of an ``out_features x in_features`` packed matrix (row-major rows)."""
    elems, bb = QUANT_BLOCK_SIZES[type_id(qtype)]
    if elems != QK_K or in_features % QK_K:
        raise ValueError(f"invalid {qtype} matrix width")
    return out_features * (in_features // QK_K) * bb
