"""Packed embedding gather vs the golden rows and the oracle (reference
tests/test_embedding.py:6-18: fp16 rows bit-equal to the oracle's)."""
import numpy as np
import pytest
import torch

from conftest import bits_equal
from gpu_util import cuda, random_packed_gpu
from gsq_b200 import _lib
from gsq_b200.nn import GSQEmbedding
from gsq_b200.quant.layouts import SUPPORTED_QUANT_TYPES
from gsq_b200.runtime import PackedWeight
from gsq_b200.runtime.kernels import iq2_s_embedding, packed_embedding

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_embedding_golden_fp16(qtype, golden):
    out = packed_embedding(cuda(golden[f"{qtype}/ids"]), cuda(golden[f"{qtype}/packed"]), qtype=qtype,
                           vocab_size=4, dimensions=512, dtype=torch.float16)
    exp = golden[f"{qtype}/emb"].reshape(*golden[f"{qtype}/ids"].shape, 512)
    np.testing.assert_array_equal(out.cpu().numpy(), exp)


@pytest.mark.parametrize("qtype", SUPPORTED_QUANT_TYPES)
def test_embedding_dtypes(qtype, golden):
    ids = cuda(golden[f"{qtype}/ids"])
    deq = torch.from_numpy(golden[f"{qtype}/deq"].reshape(4, 512))
    exp = deq[torch.from_numpy(golden[f"{qtype}/ids"].reshape(-1)).long()]
    f32 = packed_embedding(ids, cuda(golden[f"{qtype}/packed"]), qtype=qtype, vocab_size=4, dimensions=512,
                           dtype=torch.float32)
    assert bits_equal(f32.cpu().numpy(), exp.numpy())
    bf = packed_embedding(ids, cuda(golden[f"{qtype}/packed"]), qtype=qtype, vocab_size=4, dimensions=512)
    assert bf.dtype == torch.bfloat16
    assert torch.equal(bf.cpu().reshape(-1, 512), exp.to(torch.bfloat16))


def test_iq2_s_vocab_248320_selected_rows(oracle_mod):
    """The reference test's ids [0, 17, 248046] on a full-vocab IQ2_S table."""
    vocab, dim = 248320, 5120
    packed = random_packed_gpu("IQ2_S", vocab, dim, seed=5)
    ids = torch.tensor([[0, 17, 248046]], dtype=torch.int32, device="cuda")
    out = iq2_s_embedding(ids, packed, vocab_size=vocab, dimensions=dim, dtype=torch.float16)
    rb = (dim // 256) * 82
    host = packed.cpu().numpy()
    exp = np.stack([oracle_mod.dequantize_c(host[t * rb:(t + 1) * rb], "IQ2_S") for t in (0, 17, 248046)])
    np.testing.assert_array_equal(out.cpu().numpy().reshape(3, dim), exp.astype(np.float16))


def test_q6k_embedding_layer(oracle_mod):
    vocab, dim = 1000, 5120
    packed = random_packed_gpu("Q6_K", vocab, dim, seed=8)
    w = PackedWeight.from_packed("token_embd.weight", packed, "Q6_K", (vocab, dim))
    layer = GSQEmbedding(w, dtype=torch.bfloat16)
    ids = torch.randint(0, vocab, (2, 7), device="cuda", dtype=torch.int32)
    out = layer(ids)
    assert out.shape == (2, 7, dim)
    rb = (dim // 256) * 210
    host = packed.cpu().numpy()
    for t in ids.reshape(-1).tolist()[:4]:
        row = oracle_mod.dequantize_c(host[t * rb:(t + 1) * rb], "Q6_K")
        got = out.reshape(-1, dim)[ids.reshape(-1).tolist().index(t)]
        assert torch.equal(got.cpu(), torch.from_numpy(row).to(torch.bfloat16))


def test_embedding_out_of_range_reports():
    packed = random_packed_gpu("Q4_K", 4, 256, seed=2)
    packed_embedding(torch.tensor([0, 9], dtype=torch.int32, device="cuda"), packed, qtype="Q4_K", vocab_size=4,
                     dimensions=256)
    assert _lib.load().gsq_device_status(_lib.stream_ptr(torch.device("cuda"))) == 2
    assert _lib.load().gsq_device_status(_lib.stream_ptr(torch.device("cuda"))) == 0
