"""CPU oracle for the packed-GGUF hot path (numpy + the C restatement).

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module; only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use it, as the checker.

Pinning.  The reference's decoder of record is
``mlx_gsq/quant/reference.py:10-18`` (``dequantize_reference``), a thin wrapper
over the third-party gguf-py package, pinned here to gguf 0.19.0 (the version
installed in this image; the reference's ``pyproject.toml:13`` asks for
``gguf>=0.17`` and vendors nothing).  The functions below restate gguf-py's
published ``dequantize_blocks`` algorithms (``gguf/quants.py`` line numbers are
cited per type) in float32 with the same operation order, so their output is
bit-identical.  They are checked bit-for-bit against golden vectors that the
reference's own ``dequantize_reference`` produced (``tests/golden/``,
generator ``tests/golden/make_golden.py``) and against gguf-py live.

The expected QMV/QMM value is the reference tests' ``x @ deq.T``
(``tests/test_all_qmv.py:22``, ``tests/test_all_qmm.py:34-35``), here in float64.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(REPO, "mlx-gsq-rco_b200"))

from gsq_b200.quant.layouts import LAYOUTS, QK_K, type_id  # noqa: E402
from gsq_b200.quant import tables  # noqa: E402

f32 = np.float32


def _h(blocks, off):
    """fp16 field at byte ``off`` of every block, as float32."""
    return blocks[:, off:off + 2].copy().view(np.float16).astype(f32).reshape(-1)


def _u16(blocks, off, count):
    return blocks[:, off:off + 2 * count].copy().view(np.uint16).reshape(len(blocks), count)


def _u32(blocks, off, count):
    return blocks[:, off:off + 4 * count].copy().view(np.uint32).reshape(len(blocks), count)


def _signed(v, bits):
    """Multiply by +1/-1 according to bit j of ``bits`` (gguf-py np.where signs)."""
    return v * np.where(bits != 0, f32(-1), f32(1))


def _bits8(byte_arr):
    """(..., ) uint8 -> (..., 8) bit planes."""
    return (byte_arr[..., None] >> np.arange(8, dtype=np.uint8)) & np.uint8(1)


# --- K-quants ---------------------------------------------------------------

def deq_q2_k(b):  # gguf-py quants.py:404-428
    n = len(b)
    sc = b[:, 0:16]
    qs = b[:, 16:80].reshape(n, 2, 1, 32)
    d, dmin = _h(b, 80)[:, None], _h(b, 82)[:, None]
    dl = (d * (sc & 15).astype(f32))[:, :, None]           # (n,16,1)
    ml = (dmin * (sc >> 4).astype(f32))[:, :, None]
    q = (qs >> (np.arange(4, dtype=np.uint8) * 2).reshape(1, 1, 4, 1)) & np.uint8(3)
    q = q.reshape(n, 16, 16).astype(f32)
    return (dl * q - ml).reshape(n, QK_K)


def _q4k_scale_min(s):  # gguf-py quants.py:479-501
    lo, mi, hi = s[:, 0:4], s[:, 4:8], s[:, 8:12]
    sc = np.concatenate([lo & 63, (hi & 15) | ((lo >> 2) & 48)], axis=1)
    mn = np.concatenate([mi & 63, (hi >> 4) | ((mi >> 2) & 48)], axis=1)
    return sc, mn


def deq_q4_k(b):  # gguf-py quants.py:503-522
    n = len(b)
    d, dmin = _h(b, 0)[:, None], _h(b, 2)[:, None]
    sc, mn = _q4k_scale_min(b[:, 4:16])
    dl = (d * sc.astype(f32))[:, :, None]
    dm = (dmin * mn.astype(f32))[:, :, None]
    qs = b[:, 16:144].reshape(n, 4, 1, 32) >> np.array([0, 4], dtype=np.uint8).reshape(1, 1, 2, 1)
    q = (qs & np.uint8(15)).reshape(n, 8, 32).astype(f32)
    return (dl * q - dm).reshape(n, QK_K)


def deq_q6_k(b):  # gguf-py quants.py:552-572
    n = len(b)
    ql = b[:, 0:128].reshape(n, 2, 1, 64) >> np.array([0, 4], dtype=np.uint8).reshape(1, 1, 2, 1)
    ql = (ql & np.uint8(15)).reshape(n, 8, 32)
    qh = b[:, 128:192].reshape(n, 2, 1, 32) >> (np.arange(4, dtype=np.uint8) * 2).reshape(1, 1, 4, 1)
    qh = (qh & np.uint8(3)).reshape(n, 8, 32)
    q = ((ql | (qh << np.uint8(4))).astype(np.int8) - np.int8(32)).reshape(n, 16, 16).astype(f32)
    sc = b[:, 192:208].view(np.int8).astype(f32)
    dl = (_h(b, 208)[:, None] * sc)[:, :, None]
    return (dl * q).reshape(n, QK_K)


def deq_iq4_xs(b):  # gguf-py quants.py:1351-1377
    n = len(b)
    d = _h(b, 0)[:, None]
    sh = _u16(b, 2, 1)
    sl = b[:, 4:8][:, :, None] >> np.array([0, 4], dtype=np.uint8)
    sl = sl.reshape(n, 8) & np.uint8(15)
    shv = ((sh >> (np.arange(8, dtype=np.uint16) * 2)).astype(np.uint8) & np.uint8(3))
    scale = (sl | (shv << np.uint8(4))).astype(np.int8) - np.int8(32)
    dl = (d * scale.astype(f32))[:, :, None]
    qs = b[:, 8:136].reshape(n, 8, 1, 16) >> np.array([0, 4], dtype=np.uint8).reshape(1, 1, 2, 1)
    qs = (qs & np.uint8(15)).reshape(n, 8, 32)
    kv = tables.kvalues().astype(f32)[qs]
    return (dl * kv).reshape(n, QK_K)


# --- IQ lookup types ---------------------------------------------------------

def deq_iq2_xxs(b):  # gguf-py quants.py:800-828
    n = len(b)
    d = _h(b, 0)[:, None]
    words = _u32(b, 2, 16).reshape(n, 8, 2)
    aux = words[:, :, 1]
    db = (d * (f32(0.5) + (aux >> 28).astype(f32)) * f32(0.25))[:, :, None, None]
    sidx = (aux[:, :, None] >> (np.arange(4, dtype=np.uint32) * 7)) & np.uint32(127)
    signs = _bits8(tables.ksigns()[sidx])                   # (n,8,4,8)
    gidx = words[:, :, 0:1].copy().view(np.uint8).reshape(n, 8, 4)
    g = tables.grid("IQ2_XXS")[gidx]                        # (n,8,4,8)
    return _signed(db * g, signs).reshape(n, QK_K)


def deq_iq2_xs(b):  # gguf-py quants.py:870-898
    n = len(b)
    d = _h(b, 0)[:, None]
    qs = _u16(b, 2, 32)
    sc = (b[:, 66:74][:, :, None] >> np.array([0, 4], dtype=np.uint8)).reshape(n, 16) & np.uint8(15)
    db = (d * (f32(0.5) + sc) * f32(0.25)).reshape(n, 16, 1, 1)
    signs = _bits8(tables.ksigns()[qs >> 9]).reshape(n, 16, 2, 8)
    g = tables.grid("IQ2_XS")[qs & np.uint16(511)].reshape(n, 16, 2, 8)
    return _signed(db * g, signs).reshape(n, QK_K)


def deq_iq2_s(b):  # gguf-py quants.py:972-1002
    n = len(b)
    d = _h(b, 0)[:, None]
    qs = b[:, 2:34].astype(np.uint16)
    sgn = b[:, 34:66]
    qh = b[:, 66:74]
    sc = (b[:, 74:82][:, :, None] >> np.array([0, 4], dtype=np.uint8)).reshape(n, 16) & np.uint8(15)
    db = (d * (f32(0.5) + sc) * f32(0.25)).reshape(n, 16, 1, 1)
    hi = ((qh[:, :, None] >> (np.arange(4, dtype=np.uint8) * 2)) & np.uint8(3)).reshape(n, 32)
    idx = qs | (hi.astype(np.uint16) << np.uint16(8))
    g = tables.grid("IQ2_S")[idx].reshape(n, 16, 2, 8)
    signs = _bits8(sgn).reshape(n, 16, 2, 8)
    return _signed(db * g, signs).reshape(n, QK_K)


def deq_iq3_xxs(b):  # gguf-py quants.py:1026-1054
    n = len(b)
    d = _h(b, 0)[:, None]
    qs = b[:, 2:66]
    aux = _u32(b, 66, 8)
    db = (d * (f32(0.5) + (aux >> 28).astype(f32)) * f32(0.5))[:, :, None, None]
    sidx = (aux[:, :, None] >> (np.arange(4, dtype=np.uint32) * 7)) & np.uint32(127)
    signs = _bits8(tables.ksigns()[sidx])
    g = tables.grid("IQ3_XXS")[qs].reshape(n, 8, 4, 8)
    return _signed(db * g, signs).reshape(n, QK_K)


def deq_iq3_s(b):  # gguf-py quants.py:1094-1125
    n = len(b)
    d = _h(b, 0)[:, None]
    qs = b[:, 2:66].astype(np.uint16)
    qh = b[:, 66:74]
    sgn = b[:, 74:106]
    sc = (b[:, 106:110][:, :, None] >> np.array([0, 4], dtype=np.uint8)).reshape(n, 8) & np.uint8(15)
    db = (d * (1 + 2 * sc)).reshape(n, 8, 1, 1)
    hbit = _bits8(qh).reshape(n, 64).astype(np.uint16)
    idx = qs | (hbit << np.uint16(8))
    g = tables.grid("IQ3_S")[idx].reshape(n, 8, 4, 8)
    signs = _bits8(sgn).reshape(n, 8, 4, 8)
    return _signed(db * g, signs).reshape(n, QK_K)


def deq_iq1_s(b):  # gguf-py quants.py:1265-1288
    n = len(b)
    d = _h(b, 0)[:, None]
    qs = b[:, 2:34].astype(np.uint16)
    qh = _u16(b, 34, 8)
    dl = (d * (2 * ((qh >> 12) & 7) + 1)).reshape(n, 8, 1, 1)
    delta = np.where((qh & np.uint16(0x8000)) == 0, f32(0.125), f32(-0.125)).reshape(n, 8, 1, 1)
    hi = ((qh[:, :, None] >> (np.arange(4, dtype=np.uint16) * 3)) & np.uint16(7)).reshape(n, 32)
    idx = qs | (hi << np.uint16(8))
    g = tables.grid("IQ1_S")[idx].reshape(n, 8, 4, 8)
    return (dl * (g + delta)).reshape(n, QK_K)


def deq_iq1_m(b):  # gguf-py quants.py:1298-1327
    n = len(b)
    qs = b[:, 0:32].astype(np.uint16)
    qh = b[:, 32:48]
    w = _u16(b, 48, 4)
    dbits = (((w[:, 0] & 0xF000) >> 12) | ((w[:, 1] & 0xF000) >> 8) |
             ((w[:, 2] & 0xF000) >> 4) | (w[:, 3] & 0xF000)).astype(np.uint16)
    d = dbits.view(np.float16).astype(f32)[:, None]
    sc = ((w[:, :, None] >> (np.arange(4, dtype=np.uint16) * 3)) & np.uint16(7)).reshape(n, 16)
    dl = (d * (2 * sc + 1)).reshape(n, 16, 1)
    hn = ((qh[:, :, None] >> np.array([0, 4], dtype=np.uint8)) & np.uint8(15)).reshape(n, 32)
    idx = qs | ((hn & 7).astype(np.uint16) << np.uint16(8))
    delta = np.where((hn & 8) == 0, f32(0.125), f32(-0.125)).reshape(n, 16, 2, 1)
    g = tables.grid("IQ1_M")[idx].reshape(n, 16, 2, 8)
    return (dl[:, :, :, None] * (g + delta)).reshape(n, QK_K)


NUMPY_DECODERS = {
    "Q2_K": deq_q2_k, "Q4_K": deq_q4_k, "Q6_K": deq_q6_k, "IQ4_XS": deq_iq4_xs,
    "IQ2_XXS": deq_iq2_xxs, "IQ2_XS": deq_iq2_xs, "IQ2_S": deq_iq2_s,
    "IQ3_XXS": deq_iq3_xxs, "IQ3_S": deq_iq3_s, "IQ1_S": deq_iq1_s, "IQ1_M": deq_iq1_m,
}


def dequantize(packed, qtype: str) -> np.ndarray:
    """Flat float32 dequant (numpy restatement), like ``dequantize_reference``."""
    bb = LAYOUTS[qtype].block_bytes
    raw = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8).reshape(-1))
    if raw.size % bb:
        raise ValueError(f"{qtype} payload size {raw.size} is not divisible by {bb}")
    return NUMPY_DECODERS[qtype](raw.reshape(-1, bb)).astype(f32, copy=False).reshape(-1)


# --- C restatement -----------------------------------------------------------

LIB_PATH = os.path.join(HERE, "_build", "libgsq_oracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile gsq_oracle.c (gcc, -ffp-contract=off, OpenMP) into oracle/_build/."""
    import subprocess
    src = os.path.join(HERE, "gsq_oracle.c")
    os.makedirs(os.path.dirname(LIB_PATH), exist_ok=True)
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math",
                               "-fopenmp", "-fPIC", "-shared", src, "-o", LIB_PATH])
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        L.oracle_dequant.argtypes = [ctypes.c_int, P, I64, P, P, P, P]
        L.oracle_matmul.argtypes = [ctypes.c_int, P, I64, P, I64, I64, P, P, P, P]
        L.oracle_embed.argtypes = [ctypes.c_int, P, I64, P, I64, I64, P, P, P, P]
        for f in (L.oracle_dequant, L.oracle_matmul, L.oracle_embed):
            f.restype = ctypes.c_int
        _lib = L
    return _lib


def _tables_for(qtype):
    g = tables.grid_int8(qtype) if qtype in tables.GRID_TYPES else np.zeros(8, np.int8)
    return (np.ascontiguousarray(g), np.ascontiguousarray(tables.ksigns()),
            np.ascontiguousarray(tables.kvalues()))


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def dequantize_c(packed, qtype: str) -> np.ndarray:
    raw = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8).reshape(-1))
    bb = LAYOUTS[qtype].block_bytes
    if raw.size % bb:
        raise ValueError("not block aligned")
    nb = raw.size // bb
    out = np.empty(nb * QK_K, dtype=f32)
    g, ks, kv = _tables_for(qtype)
    rc = lib().oracle_dequant(type_id(qtype), _p(raw), nb, _p(out), _p(g), _p(ks), _p(kv))
    assert rc == 0, rc
    return out


def matmul_c(x, packed, qtype: str, out_features: int, in_features: int) -> np.ndarray:
    """float64 ``x @ deq(W).T`` for x of shape (M, K) (any float dtype)."""
    x32 = np.ascontiguousarray(np.asarray(x, dtype=f32).reshape(-1, in_features))
    raw = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8).reshape(-1))
    M = x32.shape[0]
    y = np.empty((M, out_features), dtype=np.float64)
    g, ks, kv = _tables_for(qtype)
    rc = lib().oracle_matmul(type_id(qtype), _p(x32), M, _p(raw), out_features, in_features,
                             _p(y), _p(g), _p(ks), _p(kv))
    assert rc == 0, rc
    return y


def embed_c(ids, packed, qtype: str, vocab: int, dim: int) -> np.ndarray:
    ids32 = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
    raw = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8).reshape(-1))
    out = np.empty((ids32.size, dim), dtype=f32)
    g, ks, kv = _tables_for(qtype)
    rc = lib().oracle_embed(type_id(qtype), _p(ids32), ids32.size, _p(raw), vocab, dim, _p(out),
                            _p(g), _p(ks), _p(kv))
    assert rc == 0, rc
    return out


def matmul_reference(x, packed, qtype: str, out_features: int, in_features: int) -> np.ndarray:
    """Numpy float64 ``x @ deq.T`` (small sizes)."""
    deq = dequantize(packed, qtype).reshape(out_features, in_features).astype(np.float64)
    return np.asarray(x, dtype=np.float64).reshape(-1, in_features) @ deq.T


def rel_l2(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64).reshape(-1)
    e = np.asarray(expected, dtype=np.float64).reshape(-1)
    den = np.linalg.norm(e)
    return float(np.linalg.norm(a - e) / (den if den > 0 else 1.0))
