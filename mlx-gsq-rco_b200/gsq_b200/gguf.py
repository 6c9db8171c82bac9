"""GGUF files: reader, writer, and the lossless packed-weight container.

Mirrors the reference's ``mlx_gsq/gguf`` package (``parser.py:89-144``,
``converter.py:22-180``): a GGUF v2/v3 directory reader that validates
metadata and tensor extents without reading payloads, and a converter that
copies every tensor's packed bytes unchanged into a one-dimensional U8
safetensors tensor of an ``mlx-gsq-packed-v1`` container (with a sidecar
manifest and SHA-256 verification).  Here the payloads then go straight to
the GPU: ``GGUFReader.weight`` / ``model_weights`` read a tensor's byte range
into pinned host memory and copy it to a CUDA uint8 tensor with one
asynchronous copy, as the packed kernels expect (no repacking).

The file formats are the contract and are kept as specified: GGUF's header,
typed key/value metadata, tensor directory and alignment; safetensors' 8-byte
header length, JSON header and data offsets; the container's
``__metadata__`` keys (``format``, ``source_format``, ``architecture``,
``tensor_quantization``) and manifest layout.
"""
from __future__ import annotations

import hashlib
import json
import mmap
import os
import struct
import tempfile
from collections import defaultdict
from dataclasses import dataclass
from pathlib import Path
from typing import Any, BinaryIO

import numpy as np

from .quant.layouts import QUANT_BLOCK_SIZES, SUPPORTED_QUANT_TYPES, GGMLQuantizationType

CONTAINER_FORMAT = "mlx-gsq-packed-v1"
COPY_CHUNK = 16 << 20


class GGUFError(ValueError):
    """Malformed or unsupported GGUF file."""


# GGML tensor types: name -> (id, elements per block, bytes per block), from
# the ids and block sizes of quant.layouts (ggml's type traits).
GGML_TYPES: dict[str, tuple[int, int, int]] = {
    t.name: (int(t), *QUANT_BLOCK_SIZES[int(t)]) for t in GGMLQuantizationType if int(t) in QUANT_BLOCK_SIZES}
TYPE_BY_ID = {v[0]: k for k, v in GGML_TYPES.items()}
PACKED_IDS = {int(GGMLQuantizationType[q]) for q in SUPPORTED_QUANT_TYPES}  # the kernels' eleven types
PLAIN_TYPES = ("F32", "F16", "BF16")

# metadata value types (GGUF spec)
_SCALARS = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
_STRING, _ARRAY = 8, 9


@dataclass(frozen=True)
class TensorInfo:
    """One tensor of the directory; ``shape`` is GGUF order (fastest first),
    the logical (row-major) shape is its reverse."""
    name: str
    shape: tuple[int, ...]
    qtype: str
    qtype_id: int
    offset: int            # from the start of the data section
    absolute_offset: int   # in the file
    num_elements: int
    num_bytes: int

    @property
    def logical_shape(self) -> tuple[int, ...]:
        return tuple(reversed(self.shape))

    def as_dict(self) -> dict[str, Any]:
        return {"name": self.name, "gguf_shape": list(self.shape), "logical_shape": list(self.logical_shape),
                "quantization_type": self.qtype, "quantization_type_id": self.qtype_id, "offset": self.offset,
                "absolute_offset": self.absolute_offset, "num_elements": self.num_elements,
                "num_bytes": self.num_bytes}


class _In:
    def __init__(self, f: BinaryIO):
        self.f = f

    def take(self, n: int) -> bytes:
        b = self.f.read(n)
        if len(b) != n:
            raise GGUFError("unexpected end of file")
        return b

    def scalar(self, code: str):
        return struct.unpack("<" + code, self.take(struct.calcsize(code)))[0]

    def text(self) -> str:
        return self.take(self.scalar("Q")).decode("utf-8")

    def value(self, kind: int):
        if kind in _SCALARS:
            return self.scalar(_SCALARS[kind])
        if kind == _STRING:
            return self.text()
        if kind == _ARRAY:
            sub, n = self.scalar("I"), self.scalar("Q")
            if sub in _SCALARS and sub != 7:  # fixed-width elements in one read
                code = _SCALARS[sub]
                return list(struct.unpack(f"<{n}{code}", self.take(n * struct.calcsize(code))))
            return [self.value(sub) for _ in range(n)]
        raise GGUFError(f"unsupported metadata value type {kind}")


class GGUFReader:
    """Metadata and tensor directory of a GGUF v2/v3 file (payloads are read
    only on request)."""

    def __init__(self, path: str | Path):
        self.path = Path(path).expanduser().resolve()
        self.file_size = self.path.stat().st_size
        with self.path.open("rb") as f:
            r = _In(f)
            if f.read(4) != b"GGUF":
                raise GGUFError(f"{path}: no GGUF magic at the start of the file")
            self.version = r.scalar("I")
            if self.version not in (2, 3):
                raise GGUFError(f"unsupported GGUF version {self.version}")
            n_tensors, n_kv = r.scalar("Q"), r.scalar("Q")
            self.metadata: dict[str, Any] = {}
            for _ in range(n_kv):
                key = r.text()
                if key in self.metadata:
                    raise GGUFError(f"metadata key {key} appears twice")
                self.metadata[key] = r.value(r.scalar("I"))
            raw = []
            for _ in range(n_tensors):
                name = r.text()
                dims = tuple(r.scalar("Q") for _ in range(r.scalar("I")))
                tid, off = r.scalar("I"), r.scalar("Q")
                raw.append((name, dims, tid, off))
            align = self.metadata.get("general.alignment", 32)
            if not isinstance(align, int) or isinstance(align, bool) or align < 1:
                raise GGUFError("invalid general.alignment")
            self.alignment = align
            self.data_offset = -(-f.tell() // align) * align
        tensors, seen = [], set()
        for name, dims, tid, off in raw:
            if name in seen:
                raise GGUFError(f"tensor {name} appears twice in the directory")
            seen.add(name)
            if tid not in TYPE_BY_ID:
                raise GGUFError(f"unknown tensor type {tid} for {name}")
            qtype = TYPE_BY_ID[tid]
            _, elems, bb = GGML_TYPES[qtype]
            count = int(np.prod(dims, dtype=np.int64)) if dims else 1
            if count % elems:
                raise GGUFError(f"{name}: {count} elements is not a whole number of {qtype} blocks")
            nbytes = count // elems * bb
            start = self.data_offset + off
            if start + nbytes > self.file_size:
                raise GGUFError(f"tensor {name} extends past the end of the file")
            tensors.append(TensorInfo(name, dims, qtype, tid, off, start, count, nbytes))
        spans = sorted((t.absolute_offset, t.absolute_offset + t.num_bytes, t.name) for t in tensors)
        for (_, end, a), (start, _, b) in zip(spans, spans[1:]):
            if end > start:
                raise GGUFError(f"tensors {a} and {b} share bytes")
        self.tensors = tuple(tensors)
        self._index = {t.name: t for t in tensors}

    def __contains__(self, name: str) -> bool:
        return name in self._index

    def tensor(self, name: str) -> TensorInfo:
        return self._index[name]

    def read_bytes(self, name: str) -> np.ndarray:
        """The tensor's payload as uint8 (host memory)."""
        t = self._index[name]
        out = np.empty(t.num_bytes, dtype=np.uint8)
        with self.path.open("rb") as f:
            f.seek(t.absolute_offset)
            if f.readinto(memoryview(out)) != t.num_bytes:
                raise GGUFError(f"{name}: the file ended before the tensor's last byte")
        return out

    def weight(self, name: str, device="cuda"):
        """A ``PackedWeight`` whose ``data`` is the unmodified payload (a CUDA
        uint8 tensor: read into pinned memory, one asynchronous copy)."""
        t = self._index[name]
        return _packed_weight(name, t.shape, t.qtype, t.qtype_id, t.num_elements,
                              _to_device(self.path, t.absolute_offset, t.num_bytes, device))

    def model_weights(self, device="cuda") -> dict:
        """Every tensor by name, as ``build_qwen35`` takes them: the eleven
        packed types as ``PackedWeight``, plain tensors as fp32 arrays."""
        return _model_weights(self.tensors, lambda t: self.weight(t.name, device), device)

    def analysis(self) -> dict[str, Any]:
        dist = defaultdict(lambda: {"tensor_count": 0, "parameter_count": 0, "byte_count": 0})
        for t in self.tensors:
            row = dist[t.qtype]
            row["tensor_count"] += 1
            row["parameter_count"] += t.num_elements
            row["byte_count"] += t.num_bytes
        meta = {k: ({"kind": "array", "length": len(v)} if isinstance(v, list) and len(v) > 256 else v)
                for k, v in self.metadata.items()}
        return {"schema_version": 1,
                "source": {"path": str(self.path), "file_size": self.file_size, "gguf_version": self.version,
                           "data_offset": self.data_offset},
                "metadata": meta,
                "summary": {"total_tensors": len(self.tensors),
                            "total_parameters": sum(t.num_elements for t in self.tensors),
                            "total_tensor_bytes": sum(t.num_bytes for t in self.tensors)},
                "quantization_distribution": dict(sorted(dist.items())),
                "tensors": [t.as_dict() for t in self.tensors]}


def _to_device(path: Path, offset: int, nbytes: int, device):
    import torch
    if device is None:
        buf = np.empty(nbytes, dtype=np.uint8)
        with open(path, "rb") as f:
            f.seek(offset)
            f.readinto(memoryview(buf))
        return torch.from_numpy(buf)
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    with open(path, "rb") as f:
        f.seek(offset)
        if f.readinto(memoryview(host.numpy())) != nbytes:
            raise GGUFError("short read")
    out = torch.empty(nbytes, dtype=torch.uint8, device=device)
    out.copy_(host, non_blocking=True)
    torch.cuda.current_stream(out.device).synchronize()  # the pinned buffer is released on return
    return out


def _packed_weight(name, gguf_shape, qtype, qtype_id, numel, data):
    from .runtime.store import PackedWeight
    return PackedWeight(name=name, data=data, gguf_shape=tuple(gguf_shape),
                        logical_shape=tuple(reversed(tuple(gguf_shape))), quantization_type=qtype,
                        quantization_type_id=qtype_id, num_elements=numel, num_bytes=int(data.numel()))


def plain_tensor(weight, device=None):
    """An F32 / F16 / BF16 tensor's payload as an fp32 tensor of its logical
    shape (the values converted exactly)."""
    import torch
    q = weight.quantization_type
    if q not in PLAIN_TYPES:
        raise TypeError(f"{weight.name} is {q}; a quantized kernel is required")
    data = weight.data
    if q == "F32":
        t = data.view(torch.float32)
    elif q == "F16":
        t = data.view(torch.float16).float()
    else:
        t = data.view(torch.bfloat16).float()
    t = t.reshape(weight.logical_shape)
    return t.to(device) if device is not None else t


def _model_weights(tensors, load, device) -> dict:
    out = {}
    for t in tensors:
        w = load(t)
        out[t.name] = w if t.qtype_id in PACKED_IDS else plain_tensor(w, device)
    return out


# ---------------------------------------------------------------- writing


def _put_value(out: bytearray, v) -> None:
    if isinstance(v, bool):
        out += struct.pack("<I?", 7, v)
    elif isinstance(v, int):
        out += struct.pack("<Iq", 11, v) if v < 0 else struct.pack("<IQ", 10, v) if v >= 2 ** 32 else \
            struct.pack("<II", 4, v)
    elif isinstance(v, float):
        out += struct.pack("<If", 6, v)
    elif isinstance(v, str):
        raw = v.encode()
        out += struct.pack("<IQ", _STRING, len(raw)) + raw
    elif isinstance(v, (list, tuple)):
        if all(isinstance(e, str) for e in v):
            out += struct.pack("<IIQ", _ARRAY, _STRING, len(v))
            for e in v:
                raw = e.encode()
                out += struct.pack("<Q", len(raw)) + raw
        elif all(isinstance(e, int) and not isinstance(e, bool) for e in v):
            out += struct.pack("<IIQ", _ARRAY, 5, len(v)) + struct.pack(f"<{len(v)}i", *v)
        else:
            out += struct.pack("<IIQ", _ARRAY, 6, len(v)) + struct.pack(f"<{len(v)}f", *v)
    else:
        raise TypeError(f"unsupported metadata value {type(v)}")


def write_gguf(path: str | Path, tensors: dict[str, tuple[str, tuple[int, ...], bytes]],
               metadata: dict[str, Any] | None = None, alignment: int = 32) -> Path:
    """Write a GGUF v3 file.  ``tensors``: name -> (type name, logical shape
    (row-major), payload bytes).  Used to make synthetic checkpoints."""
    meta = dict(metadata or {})
    meta.setdefault("general.alignment", alignment)
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for k, v in meta.items():
        raw = k.encode()
        head += struct.pack("<Q", len(raw)) + raw
        _put_value(head, v)
    offset, payloads = 0, []
    for name, (qtype, shape, payload) in tensors.items():
        tid, elems, bb = GGML_TYPES[qtype]
        count = int(np.prod(shape, dtype=np.int64))
        if count % elems or len(payload) != count // elems * bb:
            raise ValueError(f"{name}: payload does not match {qtype} {shape}")
        raw = name.encode()
        dims = tuple(reversed(shape))
        head += struct.pack("<Q", len(raw)) + raw + struct.pack("<I", len(dims))
        head += struct.pack(f"<{len(dims)}Q", *dims) + struct.pack("<IQ", tid, offset)
        payloads.append((offset, payload))
        offset += -(-len(payload) // alignment) * alignment
    head += bytes(-len(head) % alignment)
    path = Path(path)
    with path.open("wb") as f:
        f.write(head)
        base = len(head)
        for off, payload in payloads:
            f.seek(base + off)
            f.write(payload)
        f.truncate(base + offset)
    return path


# ---------------------------------------------------------------- container


def _container_header(reader: GGUFReader) -> bytes:
    quant = {t.name: {"qtype": t.qtype, "qtype_id": t.qtype_id, "gguf_shape": list(t.shape),
                      "logical_shape": list(t.logical_shape), "num_elements": t.num_elements,
                      "block_elements": GGML_TYPES[t.qtype][1], "block_bytes": GGML_TYPES[t.qtype][2]}
             for t in reader.tensors}
    header: dict[str, Any] = {"__metadata__": {
        "format": CONTAINER_FORMAT, "source_format": "GGUF",
        "architecture": str(reader.metadata.get("general.architecture", "")),
        "note": "U8 tensors contain original GGUF packed bytes; custom kernels required",
        "tensor_quantization": json.dumps(quant, separators=(",", ":"))}}
    cursor = 0
    for t in reader.tensors:
        header[t.name] = {"dtype": "U8", "shape": [t.num_bytes], "data_offsets": [cursor, cursor + t.num_bytes]}
        cursor += t.num_bytes
    raw = json.dumps(header, ensure_ascii=False, separators=(",", ":")).encode()
    return raw + b" " * (-len(raw) % 8)


def _manifest(reader: GGUFReader, container_name: str) -> dict[str, Any]:
    return {"format": CONTAINER_FORMAT, "container": container_name,
            "source": {"path": str(reader.path), "file_size": reader.file_size, "gguf_version": reader.version,
                       "architecture": reader.metadata.get("general.architecture"),
                       "name": reader.metadata.get("general.name")},
            "tensor_count": len(reader.tensors), "tensors": {t.name: t.as_dict() for t in reader.tensors}}


def manifest_path_for(container: Path) -> Path:
    return container.with_suffix(container.suffix + ".manifest.json")


def _copy_and_hash(src: Path, dst: BinaryIO, ranges: list[tuple[str, int, int]]) -> dict[str, str]:
    """Appends each (name, offset, size) byte range of ``src`` to ``dst`` and
    returns the SHA-256 of every range: the GGUF file is memory-mapped and
    each range is read once, for the copy and the digest together."""
    digests: dict[str, str] = {}
    with src.open("rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
        view = memoryview(mm)
        try:
            for name, off, n in ranges:
                part = view[off:off + n]
                try:
                    if len(part) != n:
                        raise OSError(f"{name}: the GGUF file ends inside the tensor")
                    for c in range(0, n, COPY_CHUNK):
                        dst.write(part[c:c + COPY_CHUNK])
                    digests[name] = hashlib.sha256(part).hexdigest()
                finally:
                    part.release()
        finally:
            view.release()
    return digests


def _range_digests(path: Path, ranges: list[tuple[str, int, int]]) -> dict[str, str]:
    """SHA-256 of each (name, offset, size) byte range of a file (memory-mapped)."""
    out: dict[str, str] = {}
    with path.open("rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
        view = memoryview(mm)
        try:
            for name, off, n in ranges:
                part = view[off:off + n]
                try:
                    if len(part) != n:
                        raise OSError(f"{path.name} ends inside {name}")
                    out[name] = hashlib.sha256(part).hexdigest()
                finally:
                    part.release()
        finally:
            view.release()
    return out


def convert_gguf_to_safetensors(src: str | Path, dst: str | Path, *, overwrite: bool = False,
                                verify: bool = True) -> Path:
    """Copy every tensor's packed bytes unchanged into an ``mlx-gsq-packed-v1``
    safetensors container, the contract of ``converter.py:76-118``: the
    output appears only complete (written to a temporary file in the target
    directory, synced, then renamed over the target), a sidecar manifest
    describes every tensor, and by default every tensor is verified by
    SHA-256 (the GGUF side from the digests taken while copying, the
    container side read back) with the result recorded in the manifest."""
    reader = GGUFReader(src)
    out = Path(dst).expanduser().resolve()
    if out.exists() and not overwrite:
        raise FileExistsError(out)
    out.parent.mkdir(parents=True, exist_ok=True)
    header = _container_header(reader)
    fd, tmp_name = tempfile.mkstemp(prefix=out.name + ".", suffix=".partial", dir=out.parent)
    tmp = Path(tmp_name)
    try:
        with os.fdopen(fd, "wb") as d:
            d.write(struct.pack("<Q", len(header)) + header)
            source_digests = _copy_and_hash(reader.path, d,
                                            [(t.name, t.absolute_offset, t.num_bytes) for t in reader.tensors])
            d.flush()
            os.fsync(d.fileno())
        os.replace(tmp, out)
    except BaseException:
        tmp.unlink(missing_ok=True)
        raise
    mpath = manifest_path_for(out)
    mpath.write_text(json.dumps(_manifest(reader, out.name), ensure_ascii=False, indent=2) + "\n")
    if verify:
        _verify(reader, out, mpath, source_digests, record_hashes=True)
    return out


def read_safetensors_header(path: Path) -> tuple[dict[str, Any], int]:
    """(JSON header, offset of the data section)."""
    with path.open("rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        if n > 1 << 30:
            raise ValueError("implausible safetensors header size")
        return json.loads(f.read(n)), 8 + n


def _structure_problems(reader: GGUFReader, header: dict[str, Any], data0: int, size: int,
                        manifest: dict[str, Any]) -> list[str]:
    """Everything about the container's layout and manifest that differs from
    what the GGUF directory implies (empty when they agree)."""
    problems = []
    expected = data0 + sum(t.num_bytes for t in reader.tensors)
    if size != expected:
        problems.append(f"safetensors size {size}, expected {expected}")
    listed = manifest.get("tensors", {})
    for t in reader.tensors:
        e = header.get(t.name)
        lo_hi = e.get("data_offsets") if isinstance(e, dict) else None
        if not isinstance(e, dict) or e.get("dtype") != "U8" or e.get("shape") != [t.num_bytes] \
                or not lo_hi or lo_hi[1] - lo_hi[0] != t.num_bytes:
            problems.append(f"invalid safetensors entry for {t.name}")
        m = listed.get(t.name)
        if not m or any(m.get(k) != v for k, v in t.as_dict().items()):
            problems.append(f"manifest entry of {t.name} differs from the GGUF directory")
    return problems


def _verify(reader: GGUFReader, out: Path, mpath: Path, source_digests: dict[str, str] | None,
            record_hashes: bool) -> dict[str, Any]:
    man = json.loads(mpath.read_text())
    header, data0 = read_safetensors_header(out)
    problems = _structure_problems(reader, header, data0, out.stat().st_size, man)
    if problems:
        raise ValueError("; ".join(problems))
    if source_digests is None:
        source_digests = _range_digests(reader.path, [(t.name, t.absolute_offset, t.num_bytes)
                                                      for t in reader.tensors])
    packed = _range_digests(out, [(t.name, data0 + header[t.name]["data_offsets"][0], t.num_bytes)
                                  for t in reader.tensors])
    bad = [name for name, h in source_digests.items() if packed.get(name) != h]
    if bad:
        raise ValueError(f"container bytes differ from the GGUF ranges for {', '.join(bad)}")
    result = {"algorithm": "sha256", "status": "passed", "tensor_count": len(source_digests),
              "all_packed_bytes_identical": True, "tensor_hashes": dict(source_digests)}
    if record_hashes:
        man["verification"] = result
        mpath.write_text(json.dumps(man, ensure_ascii=False, indent=2) + "\n")
    return result


def verify_conversion(src: str | Path, container: str | Path, manifest: str | Path | None = None, *,
                      record_hashes: bool = False) -> dict[str, Any]:
    """Check a container against its GGUF source (``converter.py:129-176``):
    its size, every tensor entry and manifest entry first, then the SHA-256
    of every tensor's bytes on both sides; raises ``ValueError`` naming every
    difference found."""
    reader = GGUFReader(src)
    out = Path(container)
    return _verify(reader, out, Path(manifest) if manifest else manifest_path_for(out), None, record_hashes)


def write_model_gguf(path: str | Path, weights: dict, metadata: dict[str, Any] | None = None) -> Path:
    """Write a weights dict in the form ``build_qwen35`` takes (``PackedWeight``
    for packed tensors, float tensors for plain ones, stored as F32) to a GGUF
    file: e.g. the benchmark's random-init model as a checkpoint."""
    tensors = {}
    for name, w in weights.items():
        if hasattr(w, "quantization_type"):
            tensors[name] = (w.quantization_type, tuple(w.logical_shape),
                             w.data.reshape(-1).cpu().numpy().tobytes())
        else:
            arr = w.detach().float().cpu().numpy()
            tensors[name] = ("F32", tuple(arr.shape), arr.astype(np.float32).tobytes())
    return write_gguf(path, tensors, metadata)


def main(argv=None) -> None:
    """``python -m gsq_b200.gguf analyze|convert|verify`` (as ``mlx_gsq/gguf/__main__.py``)."""
    import argparse
    ap = argparse.ArgumentParser(prog="python -m gsq_b200.gguf")
    sub = ap.add_subparsers(dest="command", required=True)
    a = sub.add_parser("analyze")
    a.add_argument("model", type=Path)
    a.add_argument("-o", "--output", type=Path, default=Path("analysis.json"))
    c = sub.add_parser("convert")
    c.add_argument("model", type=Path)
    c.add_argument("output", type=Path)
    c.add_argument("--overwrite", action="store_true")
    c.add_argument("--no-verify", action="store_true")
    v = sub.add_parser("verify")
    v.add_argument("model", type=Path)
    v.add_argument("output", type=Path)
    args = ap.parse_args(argv)
    if args.command == "analyze":
        result = GGUFReader(args.model).analysis()
        args.output.write_text(json.dumps(result, ensure_ascii=False, indent=2) + "\n")
        print(f"validated {result['summary']['total_tensors']} tensors -> {args.output}")
    elif args.command == "convert":
        print("wrote", convert_gguf_to_safetensors(args.model, args.output, overwrite=args.overwrite,
                                                    verify=not args.no_verify))
    else:
        verify_conversion(args.model, args.output)
        print("verification passed")


if __name__ == "__main__":
    main()
