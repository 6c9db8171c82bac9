"""Host logic of the Qwen3.5-hybrid harness (no GPU): model dimensions, the
per-tensor type mix, and the row-wise join of packed projections."""
import numpy as np
import pytest

from gsq_b200.models import Qwen35Config, default_type_mix, tensor_shapes
from gsq_b200.models.qwen35 import _Packed
from gsq_b200.quant.layouts import QUANT_BLOCK_SIZES, type_id
from gsq_b200.quant.synthetic import random_matrix
from gsq_b200.runtime import PackedWeight


def test_full_model_dimensions():
    cfg = Qwen35Config()
    shapes = tensor_shapes(cfg)
    params = sum(int(np.prod(s)) for s in shapes.values())
    assert 26.8e9 < params < 27.0e9  # the 27B model
    linear = [i for i in range(64) if cfg.is_linear(i)]
    assert len(linear) == 48 and not cfg.is_linear(3) and cfg.is_linear(4)
    assert shapes["blk.0.attn_qkv.weight"] == (10240, 5120)
    assert shapes["blk.0.ssm_out.weight"] == (5120, 6144)
    assert shapes["blk.3.attn_q.weight"] == (12288, 5120)
    assert shapes["blk.3.attn_output.weight"] == (5120, 6144)
    assert cfg.rotary_dim == 64


def test_type_mix_and_packed_bytes():
    cfg = Qwen35Config()
    mix, shapes = default_type_mix(cfg), tensor_shapes(cfg)
    assert mix["token_embd.weight"] == mix["output.weight"] == "Q6_K"
    assert {mix[f"blk.{i}.ffn_down.weight"] for i in range(64)} == {"Q4_K"}
    assert {mix[f"blk.{i}.ffn_gate.weight"] for i in range(64)} == {"IQ2_XS", "IQ2_S"}
    for i in range(64):  # the joined projections of a layer share a type
        assert mix[f"blk.{i}.ffn_gate.weight"] == mix[f"blk.{i}.ffn_up.weight"]
    total = sum(s[0] * s[1] // 256 * QUANT_BLOCK_SIZES[type_id(mix[n])][1] for n, s in shapes.items() if n in mix)
    assert 12.0e9 < total < 12.5e9


def test_row_join_is_a_packed_matrix():
    import oracle
    k = 512
    a = random_matrix("IQ3_S", 48, k, seed=1)
    b = random_matrix("IQ3_S", 80, k, seed=2)
    pa = PackedWeight.from_packed("a", a, "IQ3_S", (48, k), device=None)
    pb = PackedWeight.from_packed("b", b, "IQ3_S", (80, k), device=None)
    j = _Packed([pa, pb])
    assert (j.n, j.k, j.qtype) == (128, k, "IQ3_S")
    joined = oracle.dequantize(j.data.numpy(), "IQ3_S").reshape(128, k)
    np.testing.assert_array_equal(joined[:48], oracle.dequantize(a, "IQ3_S").reshape(48, k))
    np.testing.assert_array_equal(joined[48:], oracle.dequantize(b, "IQ3_S").reshape(80, k))


def test_row_join_rejects_mixed_types():
    pa = PackedWeight.from_packed("a", random_matrix("IQ3_S", 8, 256, seed=1), "IQ3_S", (8, 256), device=None)
    pb = PackedWeight.from_packed("b", random_matrix("IQ4_XS", 8, 256, seed=1), "IQ4_XS", (8, 256), device=None)
    with pytest.raises(ValueError):
        _Packed([pa, pb])
    pc = PackedWeight.from_packed("c", random_matrix("IQ3_S", 8, 512, seed=1), "IQ3_S", (8, 512), device=None)
    with pytest.raises(ValueError):
        _Packed([pa, pc])


def test_config_check():
    with pytest.raises(ValueError):
        Qwen35Config(head_dim=128).check()
    with pytest.raises(ValueError):
        Qwen35Config(linear_num_value_heads=40, linear_num_key_heads=16).check()
    Qwen35Config().check()


def test_glue_abi_validation():
    from gsq_b200 import _lib
    lib = _lib.load()
    fake = 1 << 20  # never dereferenced: every call fails validation first
    assert lib.gsq_rmsnorm(None, None, 1, 16, fake, 1e-6, fake, 1, None) == _lib.GSQ_ERR_ARG
    assert lib.gsq_rmsnorm(fake, None, 1, 16, fake, 1e-6, fake, 9, None) == _lib.GSQ_ERR_ARG
    assert lib.gsq_silu_mul(fake, 0, 1, 0, 0, fake, 1, None) == _lib.GSQ_ERR_SIZE
    assert lib.gsq_silu_mul(fake, 0, 1, 12, 8, fake, 1, None) == _lib.GSQ_ERR_SIZE  # n not a multiple of the group
    assert lib.gsq_silu_mul(fake, 5, 1, 16, 8, fake, 1, None) == _lib.GSQ_ERR_ARG   # input dtype
    q4k = 12
    assert lib.gsq_qmv_swiglu(q4k, fake, 1, fake, 12, 256, 1, fake, 1, None, 0, None) == _lib.GSQ_ERR_SIZE
    assert lib.gsq_qmv_swiglu(q4k, fake, 1, fake, 16, 256, 8, fake, 1, None, 0, None) == _lib.GSQ_ERR_SIZE
    assert lib.gsq_gdn_scratch_bytes(1, 16, 48) == 0  # one token runs as a single kernel
    assert lib.gsq_gdn_scratch_bytes(2, 16, 48) > 0

    def gdn(proj_stride, ab, T, nv, scratch_bytes, x=None, hidden=0):
        return lib.gsq_gdn(fake, proj_stride, ab, 96, x, hidden, fake if x else None, hidden, T, 16, nv, fake, fake,
                           fake, fake, fake, fake, 1e-6, fake, fake, scratch_bytes, fake, 1, None)

    assert gdn(20000, fake, 1, 40, 1 << 30) == _lib.GSQ_ERR_SIZE  # value heads a multiple of key heads
    assert gdn(16384, fake, 4, 48, 16) == _lib.GSQ_ERR_WORKSPACE  # scratch too small
    assert gdn(16384, None, 1, 48, 0) == _lib.GSQ_ERR_ARG  # no gates and no input to form them
    assert gdn(16384, None, 1, 48, 0, x=fake + 8, hidden=5120) == _lib.GSQ_ERR_ALIGN
    assert lib.gsq_attn_decode(fake, 24, 5, fake, fake, 1e-6, 64, 1e7, fake, fake, 256, fake, fake, 1,
                               None) == _lib.GSQ_ERR_SIZE
    assert lib.gsq_attn_decode(fake, 24, 4, fake, fake, 1e-6, 65, 1e7, fake, fake, 256, fake, fake, 1,
                               None) == _lib.GSQ_ERR_SIZE


def test_interleaved_join():
    import oracle
    k = 256
    a = random_matrix("IQ2_XS", 32, k, seed=3)
    b = random_matrix("IQ2_XS", 32, k, seed=4)
    pa = PackedWeight.from_packed("gate", a, "IQ2_XS", (32, k), device=None)
    pb = PackedWeight.from_packed("up", b, "IQ2_XS", (32, k), device=None)
    j = _Packed([pa, pb], interleave=8)
    rows = oracle.dequantize(j.data.numpy(), "IQ2_XS").reshape(64, k)
    ga = oracle.dequantize(a, "IQ2_XS").reshape(32, k)
    gb = oracle.dequantize(b, "IQ2_XS").reshape(32, k)
    for t in range(4):
        np.testing.assert_array_equal(rows[16 * t:16 * t + 8], ga[8 * t:8 * t + 8])
        np.testing.assert_array_equal(rows[16 * t + 8:16 * t + 16], gb[8 * t:8 * t + 8])
    with pytest.raises(ValueError):
        _Packed([pa, PackedWeight.from_packed("c", random_matrix("IQ2_XS", 24, k, seed=5), "IQ2_XS", (24, k),
                                              device=None)], interleave=8)



def test_head_split_build_on_one_rank():
    """build_qwen35_head_split on one rank is the whole model (nothing to
    reduce); a model takes one split, by rows or by heads."""
    import torch
    from gsq_b200.models import Qwen35, build_qwen35_head_split, random_weights
    cfg = Qwen35Config(hidden_size=512, intermediate_size=1024, num_hidden_layers=4, num_attention_heads=8,
                       num_key_value_heads=2, vocab_size=256, linear_num_value_heads=24, linear_num_key_heads=8)
    w = random_weights(cfg, "cpu", seed=2)
    m = build_qwen35_head_split(w, cfg, "cpu", max_len=16)
    assert m.reduce_group is None and m.cfg == cfg
    for L, i in zip(m.layers, range(cfg.num_hidden_layers)):
        p = f"blk.{i}."
        if L["linear"]:
            assert torch.equal(L["qkvz"].data[:w[p + "attn_qkv.weight"].num_bytes], w[p + "attn_qkv.weight"].data)
    with pytest.raises(ValueError):
        Qwen35(w, cfg, "cpu", group=object(), reduce_group=object())
