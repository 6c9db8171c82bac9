"""Fused dequantize + matvec (gsq_qmv) vs the oracle's x @ deq.T.

Primary bar: rel-L2 <= 1e-3 (fp32 accumulate).  Mirrors the reference's
tests/test_all_qmv.py:9-24 (rows 2 and 5, N=4, fp32 x) on the golden
fixtures, then widens to ragged shapes, every activation dtype, the
single-matvec benchmark matrix (Q4_K 5120x5120) and the full-size sweep
shapes (11 types x 5120->5120, 5120->17408, 17408->5120)."""
import numpy as np
import pytest
import torch

from gpu_util import REL_L2, cuda, dense_gpu, random_packed_gpu, rel_l2
from gsq_b200.quant.layouts import SUPPORTED_QUANT_TYPES
from gsq_b200.quant.synthetic import random_activations, random_matrix
from gsq_b200.runtime.kernels import quantized_matvec

pytestmark = pytest.mark.gpu

N, K = 4, 512


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
@pytest.mark.parametrize("rows", [1, 2, 5])
def test_qmv_golden(qtype, rows, golden):
    x = cuda(golden[f"x{rows}"].astype(np.float32))
    y = quantized_matvec(x, cuda(golden[f"{qtype}/packed"]), qtype=qtype, out_features=N, in_features=K)
    exp = golden[f"{qtype}/y{rows}"]
    assert y.dtype == torch.float32 and y.shape == (rows, N)
    assert rel_l2(y.cpu(), exp) <= REL_L2
    # elementwise, scaled to the output magnitude (synthetic weights are large)
    np.testing.assert_allclose(y.cpu().numpy(), exp, rtol=1e-3, atol=1e-3 * np.abs(exp).max())


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
@pytest.mark.parametrize("shape", [(64, 512), (200, 1024), (1000, 4096), (130, 256)])
@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16, torch.float32])
def test_qmv_shapes_dtypes(qtype, shape, xdt, oracle_mod):
    n, k = shape
    packed = random_matrix(qtype, n, k, seed=n + k)
    for rows in (1, 3):
        x = torch.from_numpy(random_activations(rows, k, seed=rows)).to(xdt)
        y = quantized_matvec(x.cuda(), cuda(packed), qtype=qtype, out_features=n, in_features=k,
                             out_dtype=torch.float32)
        exp = oracle_mod.matmul_c(x.float().numpy(), packed, qtype, n, k)
        assert rel_l2(y.cpu(), exp) <= REL_L2, (qtype, shape, xdt, rows)


def test_qmv_output_dtype_follows_input(golden):
    x = cuda(golden["x1"])  # fp16
    y = quantized_matvec(x, cuda(golden["Q4_K/packed"]), qtype="Q4_K", out_features=N, in_features=K)
    assert y.dtype == torch.float16
    assert rel_l2(y.float().cpu(), golden["Q4_K/y1"]) <= 2e-3


def test_qmv_config1_q4k_5120(oracle_mod):
    """The single-matvec benchmark case: Q4_K 5120x5120, seed 0, fp16 x N(0,1), fp32 y."""
    packed = random_matrix("Q4_K", 5120, 5120, seed=0)
    x = random_activations(1, 5120, seed=0, dtype=np.float16)
    y = quantized_matvec(cuda(x), cuda(packed), qtype="Q4_K", out_features=5120, in_features=5120,
                         out_dtype=torch.float32)
    exp = oracle_mod.matmul_c(x.astype(np.float32), packed, "Q4_K", 5120, 5120)
    assert rel_l2(y.cpu(), exp) <= REL_L2


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
@pytest.mark.parametrize("nk", [(5120, 5120), (17408, 5120), (5120, 17408)])
def test_qmv_config2_full_size(qtype, nk):
    """Config-2 shapes: compare with the (bit-exact) GPU dequant + fp64 matmul."""
    n, k = nk
    packed = random_packed_gpu(qtype, n, k, seed=n ^ k)
    x = torch.randn(1, k, device="cuda", dtype=torch.float16)
    y = quantized_matvec(x, packed, qtype=qtype, out_features=n, in_features=k, out_dtype=torch.float32)
    exp = x.double() @ dense_gpu(packed, qtype, n, k).T
    assert rel_l2(y.cpu(), exp.cpu()) <= REL_L2


def test_qmv_deterministic():
    packed = random_packed_gpu("IQ2_XS", 5120, 17408, seed=3)
    x = torch.randn(1, 17408, device="cuda", dtype=torch.float16)
    a = quantized_matvec(x, packed, qtype="IQ2_XS", out_features=5120, in_features=17408, out_dtype=torch.float32)
    b = quantized_matvec(x, packed, qtype="IQ2_XS", out_features=5120, in_features=17408, out_dtype=torch.float32)
    assert torch.equal(a, b)


def test_qmv_zero_activation():
    packed = random_packed_gpu("Q6_K", 256, 1024, seed=1)
    y = quantized_matvec(torch.zeros(1, 1024, device="cuda"), packed, qtype="Q6_K", out_features=256,
                         in_features=1024)
    assert torch.count_nonzero(y) == 0


def _outlier_activations(k: int, seed: int) -> torch.Tensor:
    """fp16 activations shaped like post-RMSNorm rows with outlier channels:
    N(0,1) values, in every 32-group one channel 1000x larger, some groups
    entirely tiny (1e-3 scale) and one group all zero."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(k // 32, 32, generator=g, dtype=torch.float64)
    ch = torch.randint(0, 32, (k // 32,), generator=g)
    sign = torch.where(torch.rand(k // 32, generator=g, dtype=torch.float64) < 0.5, -1.0, 1.0)
    x[torch.arange(k // 32), ch] = sign * 1000.0 * (1.0 + torch.rand(k // 32, generator=g, dtype=torch.float64))
    tiny = torch.randperm(k // 32, generator=g)[:8]
    x[tiny] = torch.randn(8, 32, generator=g, dtype=torch.float64) * 1e-3
    x[int(torch.randperm(k // 32, generator=g)[0])] = 0.0
    return x.reshape(1, k).to(torch.float16).cuda()


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_qmv_outlier_activations(qtype):
    """The matvec quantises each 32-group of x to 16-bit fixed point against
    the group's max |x|; activations with a 1000x outlier channel in every
    group, all-tiny groups and an all-zero group are held to the same bar,
    rel-L2 <= 1e-3 against the float64 product with the bit-exact dequant."""
    n = k = 5120
    packed = random_packed_gpu(qtype, n, k, seed=77)
    x = _outlier_activations(k, seed=5)
    y = quantized_matvec(x, packed, qtype=qtype, out_features=n, in_features=k, out_dtype=torch.float32)
    exp = x.double() @ dense_gpu(packed, qtype, n, k).T
    assert torch.isfinite(y).all()
    assert rel_l2(y.cpu(), exp.cpu()) <= REL_L2
