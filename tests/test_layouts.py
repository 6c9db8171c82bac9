"""Block layouts, type ids and codebooks against the reference's tables."""
import ast
import os

import numpy as np
import pytest

from gsq_b200.quant import tables
from gsq_b200.quant.layouts import (LAYOUTS, QUANT_BLOCK_SIZES, SUPPORTED_QUANT_TYPES, GGMLQuantizationType,
                                    packed_bytes)
from gsq_b200.quant.synthetic import SCALE_HI, SCALE_LO, random_blocks, random_matrix

# The reference checkout: GSQ_REFERENCE, else a "reference" directory next to this repository.
REF = os.environ.get("GSQ_REFERENCE") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")


def test_block_sizes_match_gguf():
    gguf = pytest.importorskip("gguf")
    for q in SUPPORTED_QUANT_TYPES:
        t = GGMLQuantizationType[q]
        assert QUANT_BLOCK_SIZES[int(t)] == tuple(gguf.GGML_QUANT_SIZES[gguf.GGMLQuantizationType[q]])
        assert LAYOUTS[q].block_bytes == QUANT_BLOCK_SIZES[int(t)][1]


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "mlx_gsq/gguf/parser.py")), reason="reference absent")
def test_block_sizes_match_reference_parser():
    src = open(os.path.join(REF, "mlx_gsq/gguf/parser.py")).read()
    tree = ast.parse(src)
    table = None
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and getattr(node.targets[0], "id", None) == "QUANT_BLOCK_SIZES":
            table = ast.literal_eval(node.value)
    assert table == QUANT_BLOCK_SIZES


def test_layout_fields_fill_block():
    for q, lay in LAYOUTS.items():
        end = max(off + n for _, off, n in lay.fields)
        assert end == lay.block_bytes, q
        cover = np.zeros(lay.block_bytes, int)
        for _, off, n in lay.fields:
            cover[off:off + n] += 1
        assert (cover == 1).all(), q


def test_grids_are_small_integers():
    for q in tables.GRID_TYPES:
        g = tables.grid(q)
        assert np.array_equal(g, np.round(g)) and np.abs(g).max() <= 127
    assert tables.ksigns().shape == (128,)
    assert tables.kvalues().tolist()[0] == -127


def test_synthetic_scales_in_range():
    for q in SUPPORTED_QUANT_TYPES:
        b = random_blocks(q, 1000, seed=1)
        if q == "IQ1_M":
            w = b[:, 48:56].copy().view(np.uint16).reshape(-1, 4)
            bits = ((w[:, 0] & 0xF000) >> 12) | ((w[:, 1] & 0xF000) >> 8) | ((w[:, 2] & 0xF000) >> 4) | (w[:, 3] & 0xF000)
            d = bits.astype(np.uint16).view(np.float16).astype(np.float32)
        else:
            off = {"Q2_K": 80, "Q6_K": 208}.get(q, 0)
            d = b[:, off:off + 2].copy().view(np.float16).astype(np.float32).reshape(-1)
        assert (d >= np.float16(SCALE_LO)).all() and (d <= np.float16(SCALE_HI)).all(), q


def test_packed_bytes_config_sizes():
    # Benchmark configuration sizes: Q4_K 5120^2 = 14,745,600 B; Q6_K 17408x5120 = 73,113,600 B.
    assert packed_bytes("Q4_K", 5120, 5120) == 14_745_600
    assert packed_bytes("IQ1_S", 5120, 5120) == 5_120_000
    assert packed_bytes("Q6_K", 5120, 17408) == 73_113_600
    assert random_matrix("Q4_K", 4, 512).size == packed_bytes("Q4_K", 4, 512)
    with pytest.raises(ValueError):
        packed_bytes("Q4_K", 4, 500)


def _prmt_sign_replicate(word: int) -> int:
    """prmt.b32 d, word, 0, 0xBA98: every byte becomes 0xFF if its msb is set."""
    return sum(0xFF << (8 * j) for j in range(4) if (word >> (8 * j + 7)) & 1)


def test_ksign_masks_constant_matches_ksigns():
    """gsq_fast.cuh's ksign_masks spreads the 7-bit sign index with one
    64-bit multiply and takes the parity into bit 63; for every index the
    byte masks must equal those of gguf-py's ksigns byte."""
    import re
    src = open(os.path.join(os.path.dirname(__file__), "..", "mlx-gsq-rco_b200", "csrc", "gsq_fast.cuh")).read()
    body = src[src.index("void ksign_masks("):]
    mult = int(re.search(r"\(uint64_t\)i7 \* (0x[0-9A-Fa-f]+)ull", body).group(1), 16)
    ks = tables.ksigns()
    for i7 in range(128):
        t = (i7 * mult) & ((1 << 64) - 1)
        hi = ((t >> 32) | ((bin(i7).count("1") << 31) & 0xFFFFFFFF)) & 0xFFFFFFFF
        got = _prmt_sign_replicate(t & 0xFFFFFFFF) | (_prmt_sign_replicate(hi) << 32)
        want = sum(0xFF << (8 * j) for j in range(8) if (int(ks[i7]) >> j) & 1)
        assert got == want, i7
