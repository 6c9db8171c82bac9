"""Seeded synthetic packed weights and activations.

The real 27B checkpoint is not available, so every test and benchmark runs on
random packed super-blocks in each type's native layout: every byte is drawn
uniformly from ``np.random.default_rng(seed)``, then the fp16 super-block
scales (``d``, and ``dmin`` for the K-quants) are overwritten with fp16 values
drawn uniformly from [1e-4, 4e-3].  For IQ1_M the fp16 ``d`` has no byte field
of its own: its 16 bits are written into the top nibble of each of the four
u16 scale words (gguf-py 0.19.0 ``quants.py:1304-1308``), leaving the 3-bit
sub-scales below them random.
"""
from __future__ import annotations

import numpy as np

from .layouts import LAYOUTS, QK_K, SCALE_FIELDS

SCALE_LO = 1e-4
SCALE_HI = 4e-3


def random_blocks(qtype: str, n_blocks: int, seed: int = 0, rng=None) -> np.ndarray:
    """Return ``(n_blocks, block_bytes)`` uint8 blocks of ``qtype``."""
    layout = LAYOUTS[qtype]
    rng = np.random.default_rng(seed) if rng is None else rng
    blocks = rng.integers(0, 256, size=(n_blocks, layout.block_bytes), dtype=np.uint8)
    if qtype == "IQ1_M":
        d = rng.uniform(SCALE_LO, SCALE_HI, size=n_blocks).astype(np.float16).view(np.uint16)
        words = blocks[:, 48:56].copy().view(np.uint16).reshape(n_blocks, 4)
        for i, shift in enumerate((12, 8, 4, 0)):
            nib = ((d.astype(np.uint32) << shift) & 0xF000).astype(np.uint16)
            words[:, i] = (words[:, i] & np.uint16(0x0FFF)) | nib
        blocks[:, 48:56] = words.view(np.uint8).reshape(n_blocks, 8)
        return blocks
    for off in SCALE_FIELDS[qtype]:
        d = rng.uniform(SCALE_LO, SCALE_HI, size=n_blocks).astype(np.float16)
        blocks[:, off:off + 2] = d.view(np.uint8).reshape(n_blocks, 2)
    return blocks


def random_matrix(qtype: str, out_features: int, in_features: int, seed: int = 0) -> np.ndarray:
    """Flat uint8 packed matrix: ``out_features`` rows of ``in_features/256`` blocks."""
    if in_features % QK_K:
        raise ValueError("in_features must be a multiple of 256")
    nb = out_features * (in_features // QK_K)
    return random_blocks(qtype, nb, seed=seed).reshape(-1)


def random_activations(rows: int, in_features: int, seed: int = 0, dtype=np.float16) -> np.ndarray:
    """N(0, 1) activations of shape ``(rows, in_features)``."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal(size=(rows, in_features), dtype=np.float32).astype(dtype)


def random_matrix_torch(qtype: str, out_features: int, in_features: int, seed: int = 0, device="cuda"):
    """Same distribution as ``random_matrix`` but generated on ``device`` with
    torch's RNG (used for full-size shapes; not bit-identical to the numpy one)."""
    import torch

    layout = LAYOUTS[qtype]
    nb = out_features * (in_features // QK_K)
    gen = torch.Generator(device=device).manual_seed(seed)
    blocks = torch.randint(0, 256, (nb, layout.block_bytes), dtype=torch.uint8, device=device, generator=gen)
    d = (torch.rand(nb, 2, device=device, generator=gen) * (SCALE_HI - SCALE_LO) + SCALE_LO).to(torch.float16)
    if qtype == "IQ1_M":
        bits = d[:, 0].contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
        w = blocks[:, 48:56].contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
        for i, shift in enumerate((12, 8, 4, 0)):
            w[:, i] = (w[:, i] & 0x0FFF) | ((bits << shift) & 0xF000)
        blocks[:, 48:56] = w.to(torch.int16).view(torch.uint8).reshape(nb, 8)
    else:
        dv = d.view(torch.uint8).reshape(nb, 4)
        for i, off in enumerate(SCALE_FIELDS[qtype]):
            blocks[:, off:off + 2] = dv[:, 2 * i:2 * i + 2]
    return blocks.reshape(-1)
