"""Shared helpers of the GPU parity tests."""
import numpy as np
import torch


# Primary bar of the matvec / matmul: rel-L2 <= 1e-3 against the float64
# dequantize-then-matmul of the oracle.
REL_L2 = 1e-3


def rel_l2(a, e) -> float:
    a = np.asarray(a, dtype=np.float64).reshape(-1)
    e = np.asarray(e, dtype=np.float64).reshape(-1)
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def random_packed_gpu(qtype: str, n_rows: int, k: int, seed: int) -> torch.Tensor:
    """Random packed matrix generated on the GPU (uniform bytes, fp16 scales in
    [1e-4, 4e-3]) -- used for full-size shapes where numpy generation is slow."""
    from gsq_b200.quant.synthetic import random_matrix_torch
    return random_matrix_torch(qtype, n_rows, k, seed=seed, device="cuda")


def dense_gpu(packed: torch.Tensor, qtype: str, n: int, k: int) -> torch.Tensor:
    """Bit-exact dequant on the GPU (verified against the oracle elsewhere), fp64."""
    from gsq_b200.runtime.kernels import decode
    return decode(packed, qtype).reshape(n, k).double()
