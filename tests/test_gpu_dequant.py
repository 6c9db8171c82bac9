"""Bit-exact CUDA dequantization vs the oracle and the reference's golden
vectors (reference tests/test_metal_decoders.py:9-23,
tests/test_safetensors_routing.py:8-22, tests/test_iq3_s_decode.py)."""
import numpy as np
import pytest
import torch

from conftest import bits_equal
from gpu_util import cuda
from gsq_b200.quant.layouts import LAYOUTS, SUPPORTED_QUANT_TYPES
from gsq_b200.quant.synthetic import random_blocks
from gsq_b200.runtime import PackedWeight
from gsq_b200.runtime.kernels import decode, decode_weight

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_decode_matches_golden(qtype, golden):
    out = decode(cuda(golden[f"{qtype}/packed"]), qtype).cpu().numpy()
    assert bits_equal(out, golden[f"{qtype}/deq"])


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_decode_matches_oracle_many_blocks(qtype, oracle_mod):
    blocks = random_blocks(qtype, 4099, seed=11)
    out = decode(cuda(blocks.reshape(-1)), qtype).cpu().numpy()
    assert bits_equal(out, oracle_mod.dequantize_c(blocks, qtype))


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_decode_raw_random_bytes(qtype, oracle_mod):
    """Random fp16 scales including inf/nan: every finite output bit-identical."""
    rng = np.random.default_rng(9)
    blocks = rng.integers(0, 256, size=(512, LAYOUTS[qtype].block_bytes), dtype=np.uint8)
    out = decode(cuda(blocks.reshape(-1)), qtype).cpu().numpy()
    assert bits_equal(out, oracle_mod.dequantize_c(blocks, qtype))


def test_decode_weight_block_count(golden):
    for qtype in SUPPORTED_QUANT_TYPES:
        packed = golden[f"{qtype}/packed"]
        w = PackedWeight.from_packed("w", packed, qtype, (4, 512))
        out = decode_weight(w, block_count=4).cpu().numpy()
        assert bits_equal(out, golden[f"{qtype}/deq"][:1024])


def test_decode_empty_and_misaligned():
    for qtype in SUPPORTED_QUANT_TYPES:
        assert decode(torch.zeros(0, dtype=torch.uint8, device="cuda"), qtype).numel() == 0
    with pytest.raises(ValueError):
        decode(torch.zeros(85, dtype=torch.uint8, device="cuda"), "Q2_K")
