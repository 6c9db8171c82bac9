"""Golden data for the GGUF reader and the packed-container converter.

Writes a small GGUF file with packed and plain tensors (gguf_fixture.gguf),
parses it with the reference's own reader and converts it with the reference's
own converter (mlx_gsq/gguf/parser.py and converter.py, loaded by file path
under a stand-in package name so that mlx_gsq/__init__.py, which imports MLX,
is not executed), and records the analysis (without the machine-specific
path) and the SHA-256 of the container and manifest tensor hashes in
gguf_golden.json.  Run where the reference checkout exists (the argument, else GSQ_REFERENCE,
else a ``reference`` directory next to this repository):

    python tests/golden/make_gguf_golden.py [/path/to/reference]
"""
import hashlib
import importlib.util
import json
import os
import sys
import tempfile
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "mlx-gsq-rco_b200"))


def load_reference_gguf(ref: Path):
    pkg = types.ModuleType("refgguf")
    pkg.__path__ = [str(ref / "mlx_gsq" / "gguf")]
    sys.modules["refgguf"] = pkg
    mods = {}
    for name in ("parser", "converter"):
        spec = importlib.util.spec_from_file_location(f"refgguf.{name}", ref / "mlx_gsq" / "gguf" / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods["parser"], mods["converter"]


def write_fixture(path: Path):
    import numpy as np
    from gsq_b200.gguf import write_gguf
    from gsq_b200.quant.synthetic import random_matrix
    tensors = {
        "token_embd.weight": ("Q6_K", (4, 256), random_matrix("Q6_K", 4, 256, seed=1).tobytes()),
        "blk.0.ffn_gate.weight": ("IQ2_XS", (8, 512), random_matrix("IQ2_XS", 8, 512, seed=2).tobytes()),
        "blk.0.attn_qkv.weight": ("IQ3_S", (2, 256), random_matrix("IQ3_S", 2, 256, seed=3).tobytes()),
        "blk.0.ssm_a": ("F32", (3,), np.array([-1.5, -0.25, -3.0], dtype=np.float32).tobytes()),
        "blk.0.attn_norm.weight": ("F16", (8,), np.linspace(0.5, 1.5, 8).astype(np.float16).tobytes()),
    }
    write_gguf(path, tensors, {"general.architecture": "qwen35", "general.name": "golden fixture",
                               "qwen35.block_count": 1, "qwen35.rope.freq_base": 10000000.0,
                               "tokenizer.ggml.tokens": ["<a>", "<b>", "<c>"],
                               "qwen35.rope.dimension_sections": [11, 11, 10, 0]})


def main(ref: str):
    parser, converter = load_reference_gguf(Path(ref))
    src = HERE / "gguf_fixture.gguf"
    write_fixture(src)
    analysis = parser.GGUFReader(src).analysis()
    analysis["source"].pop("path")
    with tempfile.TemporaryDirectory() as d:
        out = Path(d) / "fixture.safetensors"
        converter.convert_gguf_to_safetensors(src, out)
        container_sha = hashlib.sha256(out.read_bytes()).hexdigest()
        manifest = json.loads((Path(d) / "fixture.safetensors.manifest.json").read_text())
    golden = {"analysis": analysis, "container_sha256": container_sha,
              "tensor_hashes": manifest["verification"]["tensor_hashes"]}
    (HERE / "gguf_golden.json").write_text(json.dumps(golden, indent=1, sort_keys=True) + "\n")
    print("wrote", src.name, "and gguf_golden.json")


if __name__ == "__main__":
    default = os.environ.get("GSQ_REFERENCE") or str(HERE.parent.parent.parent / "reference")
    main(sys.argv[1] if len(sys.argv) > 1 else default)
