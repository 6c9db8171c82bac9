"""Run one QMV or QMM case a few times (a target for ncu captures).

    python -m gsq_b200.profile_case QTYPE N K REPS [M]

M omitted or 1: fused matvec with fp16 activations; M > 1: tiled matmul with
bf16 activations.  Weights are seeded synthetic packed blocks.
"""
from __future__ import annotations

import sys

import torch

from .quant.synthetic import random_matrix_torch
from .runtime.kernels import quantized_matmul, quantized_matvec


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    q, n, k, reps = argv[0], int(argv[1]), int(argv[2]), int(argv[3])
    m = int(argv[4]) if len(argv) > 4 else 1
    w = random_matrix_torch(q, n, k, seed=1)
    x = torch.randn(m, k, device="cuda", dtype=torch.float16 if m == 1 else torch.bfloat16)
    for _ in range(reps):
        if m == 1:
            y = quantized_matvec(x, w, qtype=q, out_features=n, in_features=k, out_dtype=torch.float32)
        else:
            y = quantized_matmul(x, w, qtype=q, out_features=n, in_features=k, out_dtype=torch.float32)
    torch.cuda.synchronize()
    print("ok", q, n, k, m, float(y.abs().sum()))


if __name__ == "__main__":
    main()
