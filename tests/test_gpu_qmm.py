"""Tiled dequantize + matmul on tcgen05 (gsq_qmm) vs the oracle.

Mirrors the reference's tests/test_all_qmm.py:41-57 (rows 8/16/33, an fp16
input case, tolerance rtol=2e-3, atol=2e-3*max|expected|) plus the primary
rel-L2 <= 1e-3 bar, ragged shapes and the prefill benchmark shapes (IQ2_XS, IQ3_S, IQ4_XS,
Q6_K at 5120->17408 and 17408->5120, 16 to 2048 tokens)."""
import numpy as np
import pytest
import torch

from gpu_util import REL_L2, cuda, dense_gpu, random_packed_gpu, rel_l2
from gsq_b200.quant.layouts import SUPPORTED_QUANT_TYPES
from gsq_b200.quant.synthetic import random_activations, random_matrix, random_matrix_torch
from gsq_b200.runtime.kernels import quantized_matmul

pytestmark = pytest.mark.gpu

N, K = 4, 512


def _check(actual, expected):
    actual = np.asarray(actual, dtype=np.float64)
    assert rel_l2(actual, expected) <= REL_L2
    np.testing.assert_allclose(actual, expected, rtol=2e-3, atol=2e-3 * np.abs(expected).max())


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
@pytest.mark.parametrize("rows", [8, 33])
def test_qmm_golden(qtype, rows, golden):
    x = cuda(golden[f"x{rows}"].astype(np.float32))
    y = quantized_matmul(x, cuda(golden[f"{qtype}/packed"]), qtype=qtype, out_features=N, in_features=K)
    _check(y.cpu(), golden[f"{qtype}/y{rows}"])


def test_qmm_fp16_input(golden):
    x = cuda(golden["x8"])  # fp16 in, fp16 out like the reference
    y = quantized_matmul(x, cuda(golden["Q4_K/packed"]), qtype="Q4_K", out_features=N, in_features=K,
                         out_dtype=torch.float32)
    _check(y.cpu(), golden["Q4_K/y8"])


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
@pytest.mark.parametrize("m", [2, 16, 33, 182])
@pytest.mark.parametrize("nk", [(128, 512), (200, 768), (384, 2048)])
def test_qmm_shapes(qtype, m, nk, oracle_mod):
    n, k = nk
    packed = random_matrix(qtype, n, k, seed=n * 7 + k)
    for xdt in (torch.bfloat16, torch.float16, torch.float32):
        x = torch.from_numpy(random_activations(m, k, seed=m)).to(xdt)
        y = quantized_matmul(x.cuda(), cuda(packed), qtype=qtype, out_features=n, in_features=k,
                             out_dtype=torch.float32)
        exp = oracle_mod.matmul_c(x.float().numpy(), packed, qtype, n, k)
        _check(y.cpu(), exp)


@pytest.mark.parametrize("qtype", ["IQ2_XS", "IQ3_S", "IQ4_XS", "Q6_K"])
@pytest.mark.parametrize("nk", [(17408, 5120), (5120, 17408)])
@pytest.mark.parametrize("m", [16, 182, 512, 2048])
def test_qmm_config3(qtype, nk, m):
    """Config 3 at full size and every token count it names (M=2048 is the
    one case with several 512-token groups per weight tile; M=182 is ragged
    against every tile width)."""
    n, k = nk
    packed = random_packed_gpu(qtype, n, k, seed=m + n)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    y = quantized_matmul(x, packed, qtype=qtype, out_features=n, in_features=k, out_dtype=torch.float32)
    exp = x.double() @ dense_gpu(packed, qtype, n, k).T
    assert rel_l2(y.cpu(), exp.cpu()) <= REL_L2


@pytest.mark.parametrize("m,nk", [(40, (640, 17408)), (600, (2048, 5120)), (12, (1000, 2048))])
def test_qmm_output_types_round_the_fp32_sums(m, nk):
    """fp16 and bf16 outputs are the fp32 result rounded once to nearest even
    (split-K and whole-K tiles, a ragged last row tile); by default the
    output has x's dtype, as the reference's quantized_matmul returns."""
    n, k = nk
    w = random_matrix_torch("IQ4_XS", n, k, seed=n)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    y32 = quantized_matmul(x, w, qtype="IQ4_XS", out_features=n, in_features=k, out_dtype=torch.float32)
    for dt in (torch.float16, torch.bfloat16):
        y = quantized_matmul(x, w, qtype="IQ4_XS", out_features=n, in_features=k, out_dtype=dt)
        assert y.dtype == dt
        assert torch.equal(y, y32.to(dt))
    assert quantized_matmul(x, w, qtype="IQ4_XS", out_features=n, in_features=k).dtype == torch.bfloat16


@pytest.mark.parametrize("n,k,m", [(5120, 2048, 2048), (2560, 5120, 4096), (17408, 512, 2048)])
def test_qmm_last_wave_split(n, k, m):
    """More tiles than SMs with a last wave at most half full (160 tiles of
    128 rows x 512 tokens on 148 SMs): full waves of whole-K tiles, then the
    remaining tiles with K split over the idle SMs; 17408 x 2048 tokens (544
    tiles, a last wave of 100) stays one launch.  Against float64, and
    repeated calls agree bit for bit."""
    packed = random_packed_gpu("IQ4_XS", n, k, seed=n + m)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16, generator=torch.Generator(device="cuda").manual_seed(4))
    y = quantized_matmul(x, packed, qtype="IQ4_XS", out_features=n, in_features=k, out_dtype=torch.float32)
    y2 = quantized_matmul(x, packed, qtype="IQ4_XS", out_features=n, in_features=k, out_dtype=torch.float32)
    exp = x.double() @ dense_gpu(packed, "IQ4_XS", n, k).T
    assert rel_l2(y.cpu(), exp.cpu()) <= REL_L2
    torch.cuda.synchronize()
    assert torch.equal(y, y2)


def test_qmm_split_k_deterministic():
    """Shapes with few row tiles split K over several CTAs; the partial tiles
    are summed in split order, so repeated calls agree bit for bit."""
    w = random_matrix_torch("IQ4_XS", 640, 17408, seed=5)
    x = torch.randn(512, 17408, device="cuda", dtype=torch.bfloat16)
    a = quantized_matmul(x, w, qtype="IQ4_XS", out_features=640, in_features=17408, out_dtype=torch.float32)
    b = quantized_matmul(x, w, qtype="IQ4_XS", out_features=640, in_features=17408, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("qtype", ["IQ2_XS", "IQ3_S", "Q6_K"])
@pytest.mark.parametrize("m", [257, 300, 600, 1300])
@pytest.mark.parametrize("nk", [(1024, 5120), (512, 2048), (4096, 2048)])
def test_qmm_two_accumulators(qtype, m, nk):
    """Token tiles of two accumulators narrower than 256 columns each (M
    above 256 and not a multiple of 512: 2x160 columns at M=600, 2x224 at
    M=1300), with several token groups, with K split over up to 8 CTAs (few
    row tiles) and without."""
    n, k = nk
    packed = random_packed_gpu(qtype, n, k, seed=m + n)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    y = quantized_matmul(x, packed, qtype=qtype, out_features=n, in_features=k, out_dtype=torch.float32)
    exp = x.double() @ dense_gpu(packed, qtype, n, k).T
    assert rel_l2(y.cpu(), exp.cpu()) <= REL_L2
