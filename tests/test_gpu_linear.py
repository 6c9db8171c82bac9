"""GSQLinear dispatch (reference mlx_gsq/nn/linear.py:15-24): one row -> fused
matvec, more rows -> tiled matmul, bias added after."""
import numpy as np
import pytest
import torch

from gpu_util import REL_L2, rel_l2
from gsq_b200.nn import GSQLinear
from gsq_b200.quant.synthetic import random_matrix
from gsq_b200.runtime import PackedWeight

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qtype", ["IQ3_S", "Q4_K", "IQ2_XS"])
def test_linear_rows_dispatch(qtype, oracle_mod):
    n, k = 320, 1024
    packed = random_matrix(qtype, n, k, seed=4)
    w = PackedWeight.from_packed("w", packed, qtype, (n, k))
    bias = torch.randn(n, device="cuda")
    lin = GSQLinear(w, bias=bias)
    for shape in [(1, k), (1, 1, k), (4, k), (2, 9, k)]:
        x = torch.randn(*shape, device="cuda")
        y = lin(x)
        assert y.shape == (*shape[:-1], n)
        exp = oracle_mod.matmul_c(x.reshape(-1, k).cpu().numpy(), packed, qtype, n, k) + bias.cpu().numpy()
        assert rel_l2(y.reshape(-1, n).cpu(), exp) <= REL_L2
