"""The C-ABI library loads, exports every entry point include/gsq_b200.h and
include/gsq_model.h declare, and validates arguments before touching the GPU
(these calls only exercise host-side validation; no kernel is launched)."""
import ctypes
import os
import re

import pytest

from gsq_b200 import _lib
from gsq_b200.quant.layouts import QUANT_BLOCK_SIZES, SUPPORTED_QUANT_TYPES, type_id

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
HEADERS = [os.path.join(INCLUDE, h) for h in ("gsq_b200.h", "gsq_model.h")]


def declared_functions():
    names = []
    for h in HEADERS:
        names += re.findall(r"GSQ_API\s+[\w\s\*]+?\b(gsq_\w+)\s*\(", open(h).read())
    return names


def test_header_declares_the_abi():
    names = declared_functions()
    assert set(names) == set(_lib.SIGNATURES), names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    nm = os.popen(f"nm -D --defined-only {_lib.LIB_PATH}").read()
    for name in declared_functions():
        assert re.search(rf"\bT {name}\b", nm), name


def test_version_and_block_info():
    lib = _lib.load()
    assert b"sm_100a" in lib.gsq_version()
    e, b = ctypes.c_int(), ctypes.c_int()
    for q in SUPPORTED_QUANT_TYPES:
        assert lib.gsq_block_info(type_id(q), ctypes.byref(e), ctypes.byref(b)) == 0
        assert (e.value, b.value) == QUANT_BLOCK_SIZES[type_id(q)]
    assert lib.gsq_block_info(2, None, None) == _lib.GSQ_ERR_QTYPE  # Q4_0 is not a hot-path type
    assert "unsupported" in _lib.last_error()


def test_validation_errors_before_any_launch():
    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)
    q4k = type_id("Q4_K")
    assert lib.gsq_qmv(2, fake, 0, fake, 16, 256, 1, fake, 0, None, 0, None) == _lib.GSQ_ERR_QTYPE
    assert lib.gsq_qmv(q4k, fake, 0, fake, 16, 300, 1, fake, 0, None, 0, None) == _lib.GSQ_ERR_SIZE
    assert lib.gsq_qmv(q4k, fake, 0, None, 16, 256, 1, fake, 0, None, 0, None) == _lib.GSQ_ERR_ARG
    assert lib.gsq_qmv(q4k, fake, 0, ctypes.c_void_p((1 << 20) + 8), 16, 256, 1, fake, 0, None, 0, None) \
        == _lib.GSQ_ERR_ALIGN
    assert lib.gsq_qmv(q4k, fake, 7, fake, 16, 256, 1, fake, 0, None, 0, None) == _lib.GSQ_ERR_ARG
    # split-K shapes need a workspace
    need = lib.gsq_qmv_workspace_size(q4k, 5120, 5120, 1)
    assert need > 0
    assert lib.gsq_qmv(q4k, fake, 1, fake, 5120, 5120, 1, fake, 0, None, 0, None) == _lib.GSQ_ERR_WORKSPACE
    assert lib.gsq_qmm(q4k, fake, 2, fake, 16, 256, 4, fake, 0, None, 0, None) == _lib.GSQ_ERR_WORKSPACE
    assert lib.gsq_qmm(q4k, fake, 2, fake, 16, 256, 4, fake, 7, None, 0, None) == _lib.GSQ_ERR_ARG  # y dtype
    assert lib.gsq_qmm(q4k, ctypes.c_void_p((1 << 20) + 4), 1, fake, 16, 256, 4, fake, 0, None, 0, None) \
        == _lib.GSQ_ERR_ALIGN
    assert lib.gsq_embed(q4k, fake, 3, fake, 10, 100, fake, 1, None) == _lib.GSQ_ERR_SIZE
    assert lib.gsq_dequant(99, fake, 1, fake, None) == _lib.GSQ_ERR_QTYPE
    # empty work is a no-op success
    assert lib.gsq_qmv(q4k, fake, 0, fake, 16, 256, 0, fake, 0, None, 0, None) == 0
    assert lib.gsq_dequant(q4k, fake, 0, fake, None) == 0


def test_workspace_sizes_are_plain_host_math():
    lib = _lib.load()
    for q in SUPPORTED_QUANT_TYPES:
        t = type_id(q)
        assert lib.gsq_qmv_workspace_size(t, 17408, 5120, 1) >= 0
        # a fixed 64 KiB ticket region, then (bf16 input) an fp16 copy of x
        assert lib.gsq_qmm_workspace_size(t, 17408, 5120, 512, 2) == 65536 + 512 * 5120 * 2
        assert lib.gsq_qmm_workspace_size(t, 17408, 5120, 512, 1) == 0


def test_gather_entry_points_validate_before_any_launch():
    """The row-parallel entry points reject bad ranks, regions, row counts and
    ranges with status codes before touching the GPU."""
    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)  # never dereferenced: every call below fails validation first
    q4k = type_id("Q4_K")
    two = (ctypes.c_void_p * 2)(1 << 20, 1 << 21)
    odd = (ctypes.c_void_p * 2)(1 << 20, (1 << 21) + 16)  # second region not 256-byte aligned

    def qmv_gather(regions, world, rank, rows=1, row0=0, n=256, ntot=512, xdt=1):
        return lib.gsq_qmv_gather(q4k, fake, xdt, fake, n, 256, rows, regions, world, rank, row0, ntot, None, 0, None)

    assert qmv_gather(two, 1, 0) == _lib.GSQ_ERR_ARG      # one rank gathers nothing
    assert qmv_gather(two, 9, 0) == _lib.GSQ_ERR_ARG      # more than 8 ranks
    assert qmv_gather(two, 2, 2) == _lib.GSQ_ERR_ARG      # rank outside the group
    assert qmv_gather(None, 2, 0) == _lib.GSQ_ERR_ARG
    assert qmv_gather(odd, 2, 0) == _lib.GSQ_ERR_ALIGN
    assert qmv_gather(two, 2, 0, rows=8) == _lib.GSQ_ERR_SIZE   # 8 rows and more: the matmul
    assert qmv_gather(two, 2, 1, row0=384) == _lib.GSQ_ERR_SIZE  # rows [384, 640) outside 512
    assert qmv_gather(two, 2, 0, xdt=7) == _lib.GSQ_ERR_ARG

    def qmm_gather(regions, world, rank, m=64, row0=0, ntot=512, ydt=0):
        return lib.gsq_qmm_gather(q4k, fake, 1, fake, 256, 256, m, regions, world, rank, row0, ntot, ydt, None, 0,
                                  None)

    assert qmm_gather(two, 9, 0) == _lib.GSQ_ERR_ARG
    assert qmm_gather(two, 2, 0, ydt=2) == _lib.GSQ_ERR_ARG  # gathered values are fp32 or fp16
    assert lib.gsq_qmm_gather_mc(q4k, fake, 1, fake, 256, 256, 64, two, None, 2, 0, 0, 512, 0, None, 0,
                                 None) == _lib.GSQ_ERR_ARG  # no multicast address
    assert qmm_gather(odd, 2, 0) == _lib.GSQ_ERR_ALIGN
    assert qmm_gather(two, 2, 0, m=0) == _lib.GSQ_ERR_SIZE
    assert qmm_gather(two, 2, 0, ntot=128) == _lib.GSQ_ERR_SIZE

    assert lib.gsq_gather_region_bytes(0, 512) == 0
    assert lib.gsq_gather_region_bytes(1, 5120) > 256 + 4 * 5120  # header, y, and the one-row inbox
    p = ctypes.c_void_p()
    assert lib.gsq_gather_region_alloc(100, ctypes.byref(p)) == _lib.GSQ_ERR_ARG  # below the header size
    assert lib.gsq_gather_region_free(None) == _lib.GSQ_OK
    assert lib.gsq_ipc_export(None, ctypes.create_string_buffer(64)) == _lib.GSQ_ERR_ARG
    assert lib.gsq_ipc_import(None, ctypes.byref(p)) == _lib.GSQ_ERR_ARG
    assert lib.gsq_ipc_close(None) == _lib.GSQ_OK


def test_batched_decode_entry_points_validate_before_any_launch():
    """gsq_gdn_batch / gsq_attn_decode_batch: a batch of 0 sequences is a
    no-op, negative or oversized batches and bad shapes are rejected with
    status codes before touching the GPU."""
    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)

    def gdn_batch(batch, nk=2, nv=6, proj_stride=2048):
        return lib.gsq_gdn_batch(fake, proj_stride, fake, 12, None, 0, None, 0, batch, nk, nv, fake, fake, fake, fake,
                                 fake, fake, 1e-6, fake, fake, 0, None)

    assert gdn_batch(0) == _lib.GSQ_OK
    assert gdn_batch(-1) == _lib.GSQ_ERR_SIZE
    assert gdn_batch(70000) == _lib.GSQ_ERR_SIZE
    assert gdn_batch(4, nv=5) == _lib.GSQ_ERR_SIZE           # value heads not a multiple of key heads
    assert gdn_batch(4, proj_stride=100) == _lib.GSQ_ERR_SIZE  # row shorter than q|k|v|z

    def attn_batch(batch, nkv=4):
        return lib.gsq_attn_decode_batch(fake, 24, nkv, fake, fake, 1e-6, 64, 1e7, fake, fake, 256, fake, fake, 1,
                                         batch, None)

    assert attn_batch(0) == _lib.GSQ_OK
    assert attn_batch(-3) == _lib.GSQ_ERR_SIZE
    assert attn_batch(2, nkv=5) == _lib.GSQ_ERR_SIZE
