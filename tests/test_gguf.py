"""GGUF reader, writer, lossless container conversion and the container
store, on CPU (the reference's tests/test_gguf.py checks the same reader and
converter on a hand-made one-tensor file; here also packed types, every
validation error, tampering, and the store's fields against the oracle)."""
import json
import struct

import numpy as np
import pytest
import torch

from gsq_b200.gguf import (CONTAINER_FORMAT, GGUFError, GGUFReader, convert_gguf_to_safetensors, plain_tensor,
                           read_safetensors_header, verify_conversion, write_gguf)
from gsq_b200.quant.synthetic import random_matrix
from gsq_b200.runtime import PackedModelStore


def _str(v: str) -> bytes:
    raw = v.encode()
    return struct.pack("<Q", len(raw)) + raw


def hand_made(path, *, version=3, dims=(2, 2), tid=0, payload=None, extra_tensor=None):
    """A GGUF file assembled byte by byte (independent of write_gguf): one
    metadata string, the alignment, one F32 tensor of 2x2."""
    n_tensors = 1 + (extra_tensor is not None)
    raw = bytearray(b"GGUF" + struct.pack("<IQQ", version, n_tensors, 2))
    raw += _str("general.architecture") + struct.pack("<I", 8) + _str("test")
    raw += _str("general.alignment") + struct.pack("<II", 4, 32)
    raw += _str("weight") + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
    raw += struct.pack("<IQ", tid, 0)
    if extra_tensor is not None:
        name, off = extra_tensor
        raw += _str(name) + struct.pack("<IQQIQ", 2, 2, 2, 0, off)
    raw += bytes(-len(raw) % 32)
    raw += payload if payload is not None else struct.pack("<4f", 1, 2, 3, 4)
    path.write_bytes(bytes(raw))
    return path


def test_reader_hand_made(tmp_path):
    r = GGUFReader(hand_made(tmp_path / "tiny.gguf"))
    t = r.tensor("weight")
    assert (r.version, r.metadata["general.architecture"], r.metadata["general.alignment"]) == (3, "test", 32)
    assert t.shape == (2, 2) and t.qtype == "F32" and t.num_bytes == 16 and t.absolute_offset % 32 == 0
    assert r.read_bytes("weight").tobytes() == struct.pack("<4f", 1, 2, 3, 4)
    a = r.analysis()
    assert a["summary"] == {"total_tensors": 1, "total_parameters": 4, "total_tensor_bytes": 16}
    assert a["quantization_distribution"]["F32"]["tensor_count"] == 1


@pytest.mark.parametrize("case", ["magic", "version", "dup_tensor", "outside", "overlap", "blocks"])
def test_reader_rejects(tmp_path, case):
    p = tmp_path / "bad.gguf"
    if case == "magic":
        p.write_bytes(b"bad")
    elif case == "version":
        hand_made(p, version=1)
    elif case == "dup_tensor":
        hand_made(p, extra_tensor=("weight", 0))
    elif case == "outside":
        hand_made(p, payload=struct.pack("<2f", 1, 2))  # 8 of 16 bytes
    elif case == "overlap":
        hand_made(p, extra_tensor=("other", 8), payload=struct.pack("<8f", *range(8)))
    elif case == "blocks":
        hand_made(p, dims=(100, 1), tid=12, payload=bytes(144))  # Q4_K needs whole 256-blocks
    with pytest.raises(GGUFError):
        GGUFReader(p)


def packed_fixture(path):
    tensors = {
        "blk.0.ffn_up.weight": ("IQ2_XS", (8, 512), random_matrix("IQ2_XS", 8, 512, seed=1).tobytes()),
        "blk.0.ffn_down.weight": ("Q4_K", (4, 256), random_matrix("Q4_K", 4, 256, seed=2).tobytes()),
        "blk.0.attn_norm.weight": ("F32", (512,), np.arange(512, dtype=np.float32).tobytes()),
        "blk.0.ssm_dt.bias": ("F16", (3,), np.array([0.5, -1, 2], dtype=np.float16).tobytes()),
    }
    write_gguf(path, tensors, {"general.architecture": "qwen35", "general.name": "fixture",
                               "qwen35.block_count": 1, "tokenizer.ggml.tokens": ["a", "b"],
                               "qwen35.rope.dimension_sections": [11, 11, 10, 0]})
    return tensors


def test_writer_reader_round_trip(tmp_path):
    src = tmp_path / "m.gguf"
    tensors = packed_fixture(src)
    r = GGUFReader(src)
    assert r.metadata["qwen35.block_count"] == 1 and r.metadata["tokenizer.ggml.tokens"] == ["a", "b"]
    assert r.metadata["qwen35.rope.dimension_sections"] == [11, 11, 10, 0]
    for name, (qtype, shape, payload) in tensors.items():
        t = r.tensor(name)
        assert t.qtype == qtype and t.logical_shape == shape
        assert r.read_bytes(name).tobytes() == payload
    w = r.weight("blk.0.ffn_up.weight", device=None)
    assert w.quantization_type_id == 17 and w.logical_shape == (8, 512) and w.gguf_shape == (512, 8)
    np.testing.assert_array_equal(plain_tensor(r.weight("blk.0.ssm_dt.bias", device=None)).numpy(),
                                  np.array([0.5, -1, 2], dtype=np.float32))


def test_convert_verify_and_store(tmp_path):
    import oracle
    src, dst = tmp_path / "m.gguf", tmp_path / "m.safetensors"
    tensors = packed_fixture(src)
    convert_gguf_to_safetensors(src, dst)
    header, data0 = read_safetensors_header(dst)
    assert header["__metadata__"]["format"] == CONTAINER_FORMAT
    assert header["__metadata__"]["architecture"] == "qwen35"
    man = json.loads((tmp_path / "m.safetensors.manifest.json").read_text())
    assert man["verification"]["status"] == "passed" and man["tensor_count"] == 4
    with pytest.raises(FileExistsError):
        convert_gguf_to_safetensors(src, dst)
    for manifest_present in (True, False):
        if not manifest_present:
            (tmp_path / "m.safetensors.manifest.json").unlink()
        store = PackedModelStore(dst, device=None)
        assert len(store) == 4 and "blk.0.ffn_up.weight" in store
        w = store.weight("blk.0.ffn_up.weight")
        assert (w.quantization_type, w.logical_shape, w.num_bytes) == ("IQ2_XS", (8, 512), 8 * 2 * 74)
        np.testing.assert_array_equal(oracle.dequantize(w.data.numpy(), "IQ2_XS"),
                                      oracle.dequantize(np.frombuffer(tensors["blk.0.ffn_up.weight"][2], np.uint8),
                                                        "IQ2_XS"))
        norm = store.materialize_plain("blk.0.attn_norm.weight")
        assert norm.dtype == torch.float32 and torch.equal(norm, torch.arange(512, dtype=torch.float32))
        with pytest.raises(TypeError):
            store.materialize_plain("blk.0.ffn_down.weight")
        mw = store.model_weights()
        assert mw["blk.0.ssm_dt.bias"].dtype == torch.float32 and hasattr(mw["blk.0.ffn_down.weight"], "data")


def test_verify_detects_tampering(tmp_path):
    src, dst = tmp_path / "m.gguf", tmp_path / "m.safetensors"
    packed_fixture(src)
    convert_gguf_to_safetensors(src, dst)
    raw = bytearray(dst.read_bytes())
    raw[-1] ^= 0xFF  # last byte of the last tensor
    dst.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="differ"):
        verify_conversion(src, dst)


def test_store_rejects_foreign_safetensors(tmp_path):
    p = tmp_path / "x.safetensors"
    head = json.dumps({"__metadata__": {"format": "pt"}, "w": {"dtype": "F32", "shape": [1],
                                                                "data_offsets": [0, 4]}}).encode()
    p.write_bytes(struct.pack("<Q", len(head)) + head + bytes(4))
    with pytest.raises(ValueError):
        PackedModelStore(p, device=None)


def test_against_reference_golden(tmp_path):
    """The fixture parsed by the reference's reader and converted by the
    reference's converter (tests/golden/make_gguf_golden.py): our analysis
    must be identical and our container byte-identical (same SHA-256)."""
    import hashlib
    from pathlib import Path
    golden_dir = Path(__file__).resolve().parent / "golden"
    golden = json.loads((golden_dir / "gguf_golden.json").read_text())
    src = golden_dir / "gguf_fixture.gguf"
    ours = GGUFReader(src).analysis()
    ours["source"].pop("path")
    assert json.loads(json.dumps(ours)) == golden["analysis"]
    dst = tmp_path / "fixture.safetensors"
    convert_gguf_to_safetensors(src, dst)
    assert hashlib.sha256(dst.read_bytes()).hexdigest() == golden["container_sha256"]
    man = json.loads((tmp_path / "fixture.safetensors.manifest.json").read_text())
    assert man["verification"]["tensor_hashes"] == golden["tensor_hashes"]


def test_cli(tmp_path, capsys):
    from gsq_b200.gguf import main
    src = tmp_path / "m.gguf"
    packed_fixture(src)
    main(["analyze", str(src), "-o", str(tmp_path / "a.json")])
    assert json.loads((tmp_path / "a.json").read_text())["summary"]["total_tensors"] == 4
    main(["convert", str(src), str(tmp_path / "m.safetensors")])
    main(["verify", str(src), str(tmp_path / "m.safetensors")])
    assert "verification passed" in capsys.readouterr().out


def test_model_checkpoint_round_trip(tmp_path):
    """Every tensor of the model (a reduced configuration, random-init on the
    host) written as a GGUF checkpoint and read back through the reader and
    through the converted container: the same names, types, shapes and bytes
    (plain tensors as fp32)."""
    from gsq_b200.gguf import write_model_gguf
    from gsq_b200.models import Qwen35Config, random_weights, tensor_shapes
    cfg = Qwen35Config(hidden_size=512, intermediate_size=768, num_hidden_layers=4, num_attention_heads=4,
                       num_key_value_heads=2, vocab_size=512, linear_num_value_heads=4, linear_num_key_heads=2)
    w = random_weights(cfg, "cpu", seed=1)
    assert set(w) == set(tensor_shapes(cfg))
    src = write_model_gguf(tmp_path / "m.gguf", w, {"general.architecture": "qwen35"})
    dst = convert_gguf_to_safetensors(src, tmp_path / "m.safetensors")
    for loaded in (GGUFReader(src).model_weights(device=None), PackedModelStore(dst, device=None).model_weights()):
        assert set(loaded) == set(w)
        for name, t in w.items():
            got = loaded[name]
            if hasattr(t, "quantization_type"):
                assert got.quantization_type == t.quantization_type and got.logical_shape == t.logical_shape
                assert torch.equal(got.data.reshape(-1), t.data.reshape(-1))
            else:
                assert got.dtype == torch.float32 and torch.equal(got, t.float()), name
