"""Failure detection of the fused row gathers on one GPU, without a fault.

Rank 0 of a two-rank split runs alone: the second region is allocated on
the same GPU and no peer ever sends into it.  The kernel's bounded wait must
run out (about a second), the kernel must return normally, the device status
must report the expired wait, and this rank's own rows must be in its
output.  Nothing traps, hangs or faults: the waits end by their own limit.
"""
import ctypes
import time

import pytest
import torch

from gsq_b200 import _lib
from gsq_b200.parallel import shard_packed
from gsq_b200.quant.layouts import type_id
from gsq_b200.quant.synthetic import random_matrix_torch
from gsq_b200.runtime.kernels import quantized_matmul, quantized_matvec

pytestmark = pytest.mark.gpu

DEV_WAIT_TIMEOUT = 1


def _region(lib, rows, ntot):
    p = ctypes.c_void_p()
    _lib.check(lib.gsq_gather_region_alloc(lib.gsq_gather_region_bytes(rows, ntot), ctypes.byref(p)))
    return p


class _Array:
    """__cuda_array_interface__ view of library-owned device memory."""

    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None}


def _own_y(region, rows, ntot):
    return torch.as_tensor(_Array(region.value + 256, (rows, ntot)), device="cuda").clone().cpu()


def _run(kind):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    qtype, n, k = ("Q4_K", 1024, 5120) if kind == "qmv" else ("IQ4_XS", 512, 5120)
    rows = 1 if kind == "qmv" else 16
    packed = random_matrix_torch(qtype, n, k, seed=4, device=dev)
    shard = shard_packed(packed, qtype, n, k, 2, 0)
    x = torch.randn(rows, k, device=dev, dtype=torch.float16 if kind == "qmv" else torch.bfloat16)
    own, peer = _region(lib, rows, n), _region(lib, rows, n)
    regions = (ctypes.c_void_p * 2)(own, peer)
    tid = type_id(qtype)
    xcode = _lib.DTYPE_CODES[x.dtype]
    if kind == "qmv":
        need = lib.gsq_qmv_workspace_size(tid, n // 2, k, rows)
    else:
        need = lib.gsq_qmm_workspace_size(tid, n // 2, k, rows, xcode)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
    lib.gsq_device_status(None)  # clear any earlier status
    t0 = time.time()
    if kind == "qmv":
        code = lib.gsq_qmv_gather(tid, x.data_ptr(), xcode, shard.data_ptr(), n // 2, k, rows, regions, 2, 0, 0, n,
                                  ws.data_ptr(), ws.numel(), None)
    else:
        code = lib.gsq_qmm_gather(tid, x.data_ptr(), xcode, shard.data_ptr(), n // 2, k, rows, regions, 2, 0, 0, n,
                                  _lib.DTYPE_CODES[torch.float32], ws.data_ptr(), ws.numel(), None)
    assert code == _lib.GSQ_OK, _lib.last_error()
    status = lib.gsq_device_status(None)
    elapsed = time.time() - t0
    y = _own_y(own, rows, n)
    for r in (own, peer):
        _lib.check(lib.gsq_gather_region_free(r))
    assert status == DEV_WAIT_TIMEOUT
    assert elapsed < 30.0
    if kind == "qmv":
        ref = quantized_matvec(x, packed, qtype=qtype, out_features=n, in_features=k, out_dtype=torch.float32).cpu()
    else:
        ref = quantized_matmul(x, packed, qtype=qtype, out_features=n, in_features=k, out_dtype=torch.float32).cpu()
    mine = slice(0, n // 2)
    err = float((y[:, mine] - ref[:, mine]).norm() / ref[:, mine].norm())
    assert err <= 1e-3
    assert float(y[:, n // 2:].abs().max()) == 0.0  # the silent peer's rows never arrived


def test_qmv_gather_wait_expires_without_peer():
    _run("qmv")


def test_qmm_gather_wait_expires_without_peer():
    _run("qmm")
