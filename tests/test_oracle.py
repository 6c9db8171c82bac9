"""The CPU oracle (numpy + C restatements of gguf-py) against the golden
vectors produced by the reference's own dequantize_reference, and against
gguf-py 0.19.0 live.  Mirrors the reference's bit-exact decoder tests
(tests/test_metal_decoders.py:9-23, tests/test_safetensors_routing.py:8-22)."""
import numpy as np
import pytest

from conftest import bits_equal
from gsq_b200.quant.layouts import LAYOUTS, SUPPORTED_QUANT_TYPES
from gsq_b200.quant.synthetic import random_blocks

N, K = 4, 512


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_numpy_oracle_matches_golden(qtype, golden, oracle_mod):
    assert bits_equal(oracle_mod.dequantize(golden[f"{qtype}/packed"], qtype), golden[f"{qtype}/deq"])


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_c_oracle_matches_golden(qtype, golden, oracle_mod):
    assert bits_equal(oracle_mod.dequantize_c(golden[f"{qtype}/packed"], qtype), golden[f"{qtype}/deq"])


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_oracles_match_gguf_live(qtype, oracle_mod):
    gguf = pytest.importorskip("gguf")
    blocks = random_blocks(qtype, 300, seed=77)
    ref = gguf.dequantize(blocks, gguf.GGMLQuantizationType[qtype]).reshape(-1)
    assert bits_equal(oracle_mod.dequantize(blocks, qtype), ref)
    assert bits_equal(oracle_mod.dequantize_c(blocks, qtype), ref)


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_oracles_on_raw_random_bytes(qtype, oracle_mod):
    """Fully random bytes (random fp16 scales, incl. inf/nan) still agree bitwise
    on every finite output; NaN outputs coincide."""
    gguf = pytest.importorskip("gguf")
    rng = np.random.default_rng(5)
    blocks = rng.integers(0, 256, size=(64, LAYOUTS[qtype].block_bytes), dtype=np.uint8)
    with np.errstate(invalid="ignore", over="ignore"):
        ref = gguf.dequantize(blocks, gguf.GGMLQuantizationType[qtype]).reshape(-1)
        assert bits_equal(oracle_mod.dequantize(blocks, qtype), ref)
    assert bits_equal(oracle_mod.dequantize_c(blocks, qtype), ref)


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
@pytest.mark.parametrize("rows", [1, 2, 5, 8, 33])
def test_oracle_matmul_matches_golden(qtype, rows, golden, oracle_mod):
    x = golden[f"x{rows}"].astype(np.float32)
    y = oracle_mod.matmul_c(x, golden[f"{qtype}/packed"], qtype, N, K)
    np.testing.assert_allclose(y, golden[f"{qtype}/y{rows}"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_oracle_embedding_matches_golden(qtype, golden, oracle_mod):
    ids = golden[f"{qtype}/ids"]
    rows = oracle_mod.embed_c(ids, golden[f"{qtype}/packed"], qtype, N, K).astype(np.float16)
    np.testing.assert_array_equal(rows.reshape(golden[f"{qtype}/emb"].shape), golden[f"{qtype}/emb"])


def test_empty_payload(oracle_mod):
    for qtype in SUPPORTED_QUANT_TYPES:
        assert oracle_mod.dequantize(np.zeros(0, np.uint8), qtype).size == 0
        assert oracle_mod.dequantize_c(np.zeros(0, np.uint8), qtype).size == 0


def test_misaligned_payload_rejected(oracle_mod):
    with pytest.raises(ValueError):
        oracle_mod.dequantize(np.zeros(83, np.uint8), "Q2_K")
