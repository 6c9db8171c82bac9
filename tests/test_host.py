"""Host-side contract of the Python operators (no GPU): the reference's
validation errors (qmv.py:540-544, qmm.py:569-580, registry.py:29-31,
embedding.py:30-32) and no silent CPU fallback."""
import numpy as np
import pytest
import torch

from gsq_b200.nn import GSQEmbedding, GSQLinear
from gsq_b200.runtime import PackedWeight
from gsq_b200.runtime.kernels import (decode, decode_weight, iq2_s_embedding, packed_embedding, quantized_matmul,
                                      quantized_matvec)
from gsq_b200.quant.synthetic import random_matrix


def _w(qtype="Q4_K", n=4, k=512):
    return PackedWeight.from_packed("w", random_matrix(qtype, n, k), qtype, (n, k), device=None)


def test_matvec_validation():
    w = _w()
    x = torch.zeros(1, 512)
    with pytest.raises(ValueError):
        quantized_matvec(x, w.data, qtype="Q4_K", out_features=4, in_features=500)
    with pytest.raises(ValueError):
        quantized_matvec(x, w.data[:-1], qtype="Q4_K", out_features=4, in_features=512)
    with pytest.raises(ValueError):
        quantized_matvec(torch.zeros(1, 256), w.data, qtype="Q4_K", out_features=4, in_features=512)
    with pytest.raises(NotImplementedError):
        quantized_matvec(x, w.data, qtype="NOPE", out_features=4, in_features=512)


def test_matmul_validation():
    w = _w()
    x = torch.zeros(8, 512)
    with pytest.raises(NotImplementedError):
        quantized_matmul(x, w.data, qtype="Q5_K", out_features=4, in_features=512)
    with pytest.raises(ValueError):
        quantized_matmul(x, w.data, qtype="Q4_K", out_features=5, in_features=512)


def test_no_cpu_fallback():
    w = _w()
    with pytest.raises(RuntimeError, match="CUDA"):
        quantized_matvec(torch.zeros(1, 512), w.data, qtype="Q4_K", out_features=4, in_features=512)
    with pytest.raises(RuntimeError, match="CUDA"):
        quantized_matmul(torch.zeros(9, 512), w.data, qtype="Q4_K", out_features=4, in_features=512)
    with pytest.raises(RuntimeError, match="CUDA"):
        decode(w.data, "Q4_K")


def test_registry_errors():
    with pytest.raises(NotImplementedError):
        decode(torch.zeros(10, dtype=torch.uint8), "Q8_0")
    plain = PackedWeight("n", torch.zeros(8, dtype=torch.uint8), (2,), (2,), "F32", 0, 2, 8)
    with pytest.raises(TypeError):
        decode_weight(plain)


def test_embedding_validation():
    packed = random_matrix("IQ2_S", 3, 512)
    t = torch.from_numpy(packed)
    with pytest.raises(ValueError):
        iq2_s_embedding(torch.zeros(2, dtype=torch.int32), t, vocab_size=3, dimensions=500)
    with pytest.raises(ValueError):
        iq2_s_embedding(torch.zeros(2, dtype=torch.int32), t[:-1], vocab_size=3, dimensions=512)
    with pytest.raises(NotImplementedError):
        packed_embedding(torch.zeros(2, dtype=torch.int32), t, qtype="Q8_0", vocab_size=3, dimensions=512)


def test_layers_wire_metadata():
    w = _w("IQ3_S", 8, 768)
    lin = GSQLinear(w)
    assert (lin.in_features, lin.out_features, lin.qtype) == (768, 8, "IQ3_S")
    emb = GSQEmbedding(w, dtype=torch.float16)
    assert (emb.num_embeddings, emb.dimensions) == (8, 768)
    with pytest.raises(NotImplementedError):
        GSQEmbedding(PackedWeight("n", torch.zeros(8, dtype=torch.uint8), (2,), (1, 2), "F32", 0, 2, 8))


def test_packed_weight_from_packed_checks_size():
    with pytest.raises(ValueError):
        PackedWeight.from_packed("w", np.zeros(10, np.uint8), "Q4_K", (4, 512), device=None)
