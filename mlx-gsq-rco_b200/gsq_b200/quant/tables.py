"""Codebook tables of the IQ formats, taken from gguf-py at run time.

The reference builds its Metal lookup tables the same way: ``grid`` from
``gguf.quants.<T>.init_grid()`` / ``.grid`` and the 128-byte ``ksigns`` table
from ``gguf.quants.IQ2_XXS.ksigns`` (``mlx_gsq/runtime/kernels/iq_lookup_decode.py:46-53``,
``iq3_s_decode.py:56-61``, ``mlx_gsq/quant/reference.py:21-27``).  IQ4_XS uses
the 16-entry non-linear ``IQ4_NL.kvalues`` table (``qmm.py:147``).  Every grid
entry is a small integer, so the tables are exact as int8.
"""
from __future__ import annotations

from functools import lru_cache

import numpy as np

GRID_TYPES = {
    # qtype: (gguf class holding the grid, entries, values per entry)
    "IQ2_XXS": ("IQ2_XXS", 256, 8),
    "IQ2_XS": ("IQ2_XS", 512, 8),
    "IQ2_S": ("IQ2_S", 1024, 8),
    "IQ3_XXS": ("IQ3_XXS", 256, 4),
    "IQ3_S": ("IQ3_S", 512, 4),
    "IQ1_S": ("IQ1_S", 2048, 8),
    "IQ1_M": ("IQ1_S", 2048, 8),  # IQ1_M shares the IQ1_S grid (gguf-py quants.py:1292-1294)
}


@lru_cache(maxsize=None)
def grid(qtype: str) -> np.ndarray:
    """``(entries, values)`` float32 codebook for an IQ type."""
    from gguf import quants
    cls_name, entries, width = GRID_TYPES[qtype]
    cls = getattr(quants, cls_name)
    cls.init_grid()
    g = np.asarray(cls.grid, dtype=np.float32).reshape(entries, width)
    g.setflags(write=False)
    return g


@lru_cache(maxsize=None)
def ksigns() -> np.ndarray:
    from gguf import quants
    k = np.frombuffer(quants.IQ2_XXS.ksigns, dtype=np.uint8).copy()
    k.setflags(write=False)
    return k


@lru_cache(maxsize=None)
def kvalues() -> np.ndarray:
    from gguf import quants
    k = np.array(quants.IQ4_NL.kvalues, dtype=np.int8)
    k.setflags(write=False)
    return k


def grid_int8(qtype: str) -> np.ndarray:
    g = grid(qtype)
    gi = g.astype(np.int8)
    assert np.array_equal(gi.astype(np.float32), g), qtype
    return gi
