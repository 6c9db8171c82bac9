"""gsq_qmv_noalloc: the allocation-free matvec entry point.

Some callers of this library cannot hand it device memory for scratch space:
a host application that runs under its own fixed memory budget, a plugin that
only ever receives raw input/output pointers, or a latency-critical loop that
must never call into an allocator.  For them gsq_qmv_noalloc runs the same
fused matvec as gsq_qmv but keeps its split-K scratch in a fixed array inside
the library.  This test calls it through the C ABI and checks it against
gsq_qmv (with a caller-owned workspace), twice in a row, because the second
call relies on the first having left the shared scratch in a clean state.

This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from gpu_util import REL_L2, rel_l2
from gsq_b200 import _lib
from gsq_b200.quant.layouts import type_id
from gsq_b200.quant.synthetic import random_matrix_torch

pytestmark = pytest.mark.gpu


def _qmv_with_workspace(lib, t, x, w, n, k, rows):
    y = torch.empty(rows, n, dtype=torch.float32, device="cuda")
    need = lib.gsq_qmv_workspace_size(t, n, k, rows)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    code = lib.gsq_qmv(t, x.data_ptr(), _lib.DTYPE_CODES[x.dtype], w.data_ptr(), n, k, rows, y.data_ptr(), 0,
                       ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device))
    assert code == 0, _lib.last_error()
    return y, need


def _qmv_noalloc(lib, t, x, w, n, k, rows):
    y = torch.empty(rows, n, dtype=torch.float32, device="cuda")
    code = lib.gsq_qmv_noalloc(t, x.data_ptr(), _lib.DTYPE_CODES[x.dtype], w.data_ptr(), n, k, rows, y.data_ptr(), 0,
                               _lib.stream_ptr(x.device))
    assert code == 0, _lib.last_error()
    return y


@pytest.mark.parametrize("qtype,n,k,rows", [
    ("Q4_K", 5120, 5120, 1),      # split over K: the scratch holds partial sums and tickets
    ("IQ2_XS", 17408, 5120, 1),
    ("IQ3_S", 5120, 17408, 2),
    ("Q6_K", 1000, 2048, 3),
])
def test_noalloc_matches_workspace_entry_point(qtype, n, k, rows):
    lib = _lib.load()
    t = type_id(qtype)
    w = random_matrix_torch(qtype, n, k, seed=n + k)
    for call in range(2):
        x = torch.randn(rows, k, device="cuda", dtype=torch.float16)
        ref, need = _qmv_with_workspace(lib, t, x, w, n, k, rows)
        got = _qmv_noalloc(lib, t, x, w, n, k, rows)
        torch.cuda.synchronize()
        assert need <= 2 * 1024 * 1024
        err = rel_l2(got.cpu(), ref.cpu())
        assert err <= REL_L2, (qtype, call, err)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    t = type_id("Q4_K")
    limit = 2 * 1024 * 1024
    fake = ctypes.c_void_p(1 << 20)
    found = None
    for n in (64, 256, 1024, 4096, 9472):
        for k in (65536, 131072, 262144):
            for rows in (1, 2, 7):
                if lib.gsq_qmv_workspace_size(t, n, k, rows) > limit:
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
