"""gsq_qmv_noalloc: the allocation-free matvec entry point.

Some callers of this library cannot hand it device memory for scratch space:
a host application that runs under its own fixed memory budget, a plugin that
only ever receives raw input/output pointers, or a latency-critical loop that
must never call into an allocator.  For them gsq_qmv_noalloc runs the same
fused matvec as gsq_qmv but keeps its split-K scratch in a fixed array inside
the library.  These tests call it through the C ABI and check it against
gsq_qmv (with a caller-owned workspace) and against the bit-exact dequantized
matrix times x in float64, twice in a row, because the second call relies on
the first having left the shared scratch in a clean state; that the calls
leave the device's free memory unchanged; and that after a bounded wait has
expired (gsq_device_status reports it) the next calls are correct again.

This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from gpu_util import REL_L2, dense_gpu, rel_l2
from gsq_b200 import _lib
from gsq_b200.parallel import shard_packed
from gsq_b200.quant.layouts import type_id
from gsq_b200.quant.synthetic import random_matrix_torch

pytestmark = pytest.mark.gpu

SCRATCH_LIMIT = 2 * 1024 * 1024  # GSQ_QMV_NOALLOC_SCRATCH_BYTES


def _qmv_with_workspace(lib, t, x, w, n, k, rows):
    y = torch.empty(rows, n, dtype=torch.float32, device="cuda")
    need = lib.gsq_qmv_workspace_size(t, n, k, rows)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    code = lib.gsq_qmv(t, x.data_ptr(), _lib.DTYPE_CODES[x.dtype], w.data_ptr(), n, k, rows, y.data_ptr(), 0,
                       ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device))
    assert code == 0, _lib.last_error()
    return y, need


def _qmv_noalloc(lib, t, x, w, n, k, rows, y=None):
    if y is None:
        y = torch.empty(rows, n, dtype=torch.float32, device="cuda")
    code = lib.gsq_qmv_noalloc(t, x.data_ptr(), _lib.DTYPE_CODES[x.dtype], w.data_ptr(), n, k, rows, y.data_ptr(), 0,
                               _lib.stream_ptr(x.device))
    assert code == 0, _lib.last_error()
    return y


def _check_pair(lib, qtype, w, n, k, rows, seed):
    """One call of each entry point on the same input: both within REL_L2 of
    the float64 result, and of each other."""
    t = type_id(qtype)
    x = torch.randn(rows, k, device="cuda", dtype=torch.float16,
                    generator=torch.Generator(device="cuda").manual_seed(seed))
    ref, need = _qmv_with_workspace(lib, t, x, w, n, k, rows)
    got = _qmv_noalloc(lib, t, x, w, n, k, rows)
    exact = (x.double() @ dense_gpu(w, qtype, n, k).T).cpu()
    torch.cuda.synchronize()
    assert rel_l2(got.cpu(), ref.cpu()) <= REL_L2
    assert rel_l2(got.cpu(), exact) <= REL_L2
    return need


@pytest.mark.parametrize("qtype,n,k,rows,split", [
    ("Q4_K", 5120, 5120, 1, True),      # tiles shared between CTAs: published pieces in the scratch
    ("IQ2_XS", 17408, 5120, 1, True),
    ("IQ3_S", 5120, 17408, 2, True),
    ("Q6_K", 1000, 8192, 3, True),
    ("IQ4_XS", 4736, 5120, 1, False),   # whole tiles per CTA on 148 SMs: no scratch at all
])
def test_noalloc_matches_workspace_entry_point(qtype, n, k, rows, split):
    lib = _lib.load()
    _lib.device_status()  # start from a clear device error word
    w = random_matrix_torch(qtype, n, k, seed=n + k)
    for call in range(2):
        need = _check_pair(lib, qtype, w, n, k, rows, seed=10 * call + rows)
        assert need <= SCRATCH_LIMIT
        if split and torch.cuda.get_device_properties(0).multi_processor_count == 148:
            assert need > 0, "this shape is meant to exercise the static scratch"
    assert _lib.device_status() == 0


def test_noalloc_allocates_nothing():
    """Back-to-back calls leave the device's free memory and torch's
    allocator untouched (the first call of the process may load the module
    and look up the array's address; it is made before measuring)."""
    lib = _lib.load()
    qtype, n, k = "Q4_K", 5120, 5120
    t = type_id(qtype)
    w = random_matrix_torch(qtype, n, k, seed=1)
    x = torch.randn(1, k, device="cuda", dtype=torch.float16)
    y = torch.empty(1, n, dtype=torch.float32, device="cuda")
    _qmv_noalloc(lib, t, x, w, n, k, 1, y)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    for _ in range(4):
        _qmv_noalloc(lib, t, x, w, n, k, 1, y)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == alloc0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    t = type_id("Q4_K")
    fake = ctypes.c_void_p(1 << 20)
    found = None
    for n in (64, 256, 1024, 4096, 9472):
        for k in (65536, 131072, 262144):
            for rows in (1, 2, 7):
                if lib.gsq_qmv_workspace_size(t, n, k, rows) > SCRATCH_LIMIT:
                    found = (n, k, rows)
                    break
            if found:
                break
        if found:
            break
    if found is None:
        pytest.skip("no candidate shape needs more than the fixed scratch")
    n, k, rows = found
    code = lib.gsq_qmv_noalloc(t, fake, 1, fake, n, k, rows, fake, 0, None)
    assert code == _lib.GSQ_ERR_WORKSPACE
    assert "scratch" in _lib.last_error()


def test_noalloc_correct_after_an_expired_wait():
    """A bounded wait is made to expire without any fault: rank 0 of a
    two-rank row gather runs alone on this GPU and its peer never sends.
    gsq_device_status() reports the expiry (and re-zeroes the library's fixed
    scratch); the next two no-alloc calls must be correct again."""
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    _lib.device_status(dev)
    qtype, n, k = "Q4_K", 1024, 5120
    packed = random_matrix_torch(qtype, n, k, seed=4, device=dev)
    shard = shard_packed(packed, qtype, n, k, 2, 0)
    x = torch.randn(1, k, device=dev, dtype=torch.float16)
    regions = []
    for _ in range(2):
        p = ctypes.c_void_p()
        _lib.check(lib.gsq_gather_region_alloc(lib.gsq_gather_region_bytes(1, n), ctypes.byref(p)))
        regions.append(p)
    arr = (ctypes.c_void_p * 2)(*regions)
    tid = type_id(qtype)
    need = lib.gsq_qmv_workspace_size(tid, n // 2, k, 1)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
    code = lib.gsq_qmv_gather(tid, x.data_ptr(), _lib.DTYPE_CODES[x.dtype], shard.data_ptr(), n // 2, k, 1, arr, 2,
                              0, 0, n, ws.data_ptr(), ws.numel(), None)
    assert code == _lib.GSQ_OK, _lib.last_error()
    assert _lib.device_status(dev) == _lib.DEV_WAIT_TIMEOUT
    for r in regions:
        _lib.check(lib.gsq_gather_region_free(r))
    w = random_matrix_torch("Q4_K", 5120, 5120, seed=9, device=dev)
    for call in range(2):
        _check_pair(lib, "Q4_K", w, 5120, 5120, 1, seed=call)
    assert _lib.device_status(dev) == 0
