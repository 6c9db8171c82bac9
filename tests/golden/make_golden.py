"""Generate tests/golden/golden.npz from the reference's own decoder.

Runs only where the reference checkout exists (``GSQ_REFERENCE``, else a
``reference`` directory next to this repository).  It loads ``mlx_gsq/quant/reference.py`` by file path (a
plain ``import mlx_gsq`` needs MLX, ``mlx_gsq/__init__.py:5``) and calls its
``dequantize_reference`` -- the decoder the reference's tests treat as ground
truth (``tests/test_metal_decoders.py:21``) -- on seeded synthetic blocks.

Contents, per quant type T:
  T/packed      uint8 (8 blocks) -- also read as a 4 x 512 matrix (2 blocks/row)
  T/deq         float32 dequantize_reference(packed, T)
  x{rows}       float16 activations shared by every type, rows in (1, 2, 5, 8, 33)
  T/y{rows}     float64 expected x @ deq.T  (reference tests' expected value,
                tests/test_all_qmv.py:22, tests/test_all_qmm.py:34-35)
  T/ids, T/emb  embedding ids into the 4-row matrix and the fp16 rows the
                reference embedding test expects (tests/test_embedding.py:15-16)
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "mlx-gsq-rco_b200"))

from gsq_b200.quant.layouts import SUPPORTED_QUANT_TYPES  # noqa: E402
from gsq_b200.quant.synthetic import random_blocks  # noqa: E402

N_BLOCKS = 8
N, K = 4, 512
ROWS = (1, 2, 5, 8, 33)


def load_reference_decoder(root: str):
    path = os.path.join(root, "mlx_gsq", "quant", "reference.py")
    spec = importlib.util.spec_from_file_location("_gsq_reference_quant", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.dequantize_reference


def main(out: str = os.path.join(HERE, "golden.npz")) -> None:
    root = os.environ.get("GSQ_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))),
                                                           "reference")
    dequantize_reference = load_reference_decoder(root)
    arrays = {}
    rng = np.random.default_rng(123)
    for rows in ROWS:
        arrays[f"x{rows}"] = rng.normal(size=(rows, K)).astype(np.float16)
    for i, qtype in enumerate(SUPPORTED_QUANT_TYPES):
        packed = random_blocks(qtype, N_BLOCKS, seed=1000 + i).reshape(-1)
        deq = np.asarray(dequantize_reference(packed, qtype), dtype=np.float32)
        arrays[f"{qtype}/packed"] = packed
        arrays[f"{qtype}/deq"] = deq
        dense = deq.reshape(N, K).astype(np.float64)
        for rows in ROWS:
            x = arrays[f"x{rows}"].astype(np.float64)
            arrays[f"{qtype}/y{rows}"] = x @ dense.T
        ids = np.array([[0, 3, 1, 3, 2]], dtype=np.int32)
        arrays[f"{qtype}/ids"] = ids
        arrays[f"{qtype}/emb"] = deq.reshape(N, K)[ids.reshape(-1)].astype(np.float16)
    np.savez_compressed(out, **arrays)
    print(out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
