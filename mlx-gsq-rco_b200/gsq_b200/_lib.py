"""ctypes binding of libgsq_b200.so (the C ABI declared in include/gsq_b200.h).

There is no CPU fallback: if the library is missing or CUDA is unavailable,
every operator raises.  Build the library with ``python mlx-gsq-rco_b200/build.py``.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libgsq_b200.so")

GSQ_OK = 0
GSQ_ERR_QTYPE = -1
GSQ_ERR_SIZE = -2
GSQ_ERR_ALIGN = -3
GSQ_ERR_ARG = -4
GSQ_ERR_CUDA = -5
GSQ_ERR_WORKSPACE = -6
GSQ_ERR_DEVICE = -7

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

# name -> (restype, argtypes)
_P, _I, _I64, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "gsq_version": (ctypes.c_char_p, []),
    "gsq_last_error": (ctypes.c_char_p, []),
    "gsq_block_info": (_I, [_I, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "gsq_dequant": (_I, [_I, _P, _I64, _P, _P]),
    "gsq_qmv_workspace_size": (_SZ, [_I, _I64, _I64, _I64]),
    "gsq_qmv": (_I, [_I, _P, _I, _P, _I64, _I64, _I64, _P, _I, _P, _SZ, _P]),
    "gsq_qmm_workspace_size": (_SZ, [_I, _I64, _I64, _I64, _I]),
    "gsq_qmm": (_I, [_I, _P, _I, _P, _I64, _I64, _I64, _P, _I, _P, _SZ, _P]),
    "gsq_embed": (_I, [_I, _P, _I64, _P, _I64, _I64, _P, _I, _P]),
    "gsq_device_status": (_I, [_P]),
    "gsq_qmv_noalloc": (_I, [_I, _P, _I, _P, _I64, _I64, _I64, _P, _I, _P]),
    "gsq_gather_region_bytes": (_SZ, [_I64, _I64]),
    "gsq_gather_region_alloc": (_I, [_SZ, ctypes.POINTER(_P)]),
    "gsq_gather_region_free": (_I, [_P]),
    "gsq_ipc_export": (_I, [_P, ctypes.c_char_p]),
    "gsq_ipc_import": (_I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    "gsq_ipc_close": (_I, [_P]),
    "gsq_qmv_gather": (_I, [_I, _P, _I, _P, _I64, _I64, _I64, ctypes.POINTER(_P), _I, _I, _I64, _I64, _P, _SZ, _P]),
    "gsq_qmm_gather": (_I, [_I, _P, _I, _P, _I64, _I64, _I64, ctypes.POINTER(_P), _I, _I, _I64, _I64, _I, _P, _SZ,
                            _P]),
    "gsq_qmm_gather_mc": (_I, [_I, _P, _I, _P, _I64, _I64, _I64, ctypes.POINTER(_P), _P, _I, _I, _I64, _I64, _I, _P,
                               _SZ, _P]),
    # include/gsq_model.h: decoder-glue kernels of the model harness
    "gsq_rmsnorm": (_I, [_P, _P, _I64, _I64, _P, ctypes.c_float, _P, _I, _P]),
    "gsq_silu_mul": (_I, [_P, _I, _I64, _I64, _I64, _P, _I, _P]),
    "gsq_qmv_swiglu": (_I, [_I, _P, _I, _P, _I64, _I64, _I64, _P, _I, _P, _SZ, _P]),
    "gsq_gdn_scratch_bytes": (_SZ, [_I64, _I64, _I64]),
    "gsq_gdn": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P,
                     ctypes.c_float, _P, _P, _SZ, _P, _I, _P]),
    "gsq_attn_decode": (_I, [_P, _I64, _I64, _P, _P, ctypes.c_float, _I64, ctypes.c_float, _P, _P, _I64, _P, _P, _I,
                             _P]),
    "gsq_gdn_batch": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P,
                           ctypes.c_float, _P, _P, _I, _P]),
    "gsq_attn_decode_batch": (_I, [_P, _I64, _I64, _P, _P, ctypes.c_float, _I64, ctypes.c_float, _P, _P, _I64, _P, _P,
                                   _I, _I64, _P]),
}

_lib = None
_lock = threading.Lock()


class GSQError(RuntimeError):
    """A C-ABI call failed (status code and message from gsq_last_error)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[gsq {code}] {message}")
        self.code = code


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library (once) and bind every entry point of the header."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(f"gsq_b200 CUDA library not built: {path} is missing "
                                   "(run python mlx-gsq-rco_b200/build.py)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    return (load().gsq_last_error() or b"").decode()


def check(code: int) -> None:
    """Translate a status code into the reference's exception contract."""
    if code == GSQ_OK:
        return
    msg = last_error()
    if code == GSQ_ERR_QTYPE:
        raise NotImplementedError(msg)
    if code == GSQ_ERR_SIZE:
        raise ValueError(msg)
    raise GSQError(code, msg)


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors must live on one CUDA device; there is no host path."""
    dev = None
    for t in tensors:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"expected a torch.Tensor, got {type(t).__name__}")
        if t.device.type != "cuda":
            raise RuntimeError("gsq_b200 runs on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("tensors on different devices")
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _Workspaces:
    """Per-device zero-initialised scratch buffers, grown on demand.

    The QMV kernel leaves its ticket counters at zero after every completed
    call, so one buffer is reused across calls on the same stream.
    """

    def __init__(self):
        self._bufs: dict[tuple[int, str], torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int, kind: str = "qmv") -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        key = (device.index, kind)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf

    def reset(self, device: torch.device) -> None:
        for (idx, _), buf in self._bufs.items():
            if idx == device.index:
                buf.zero_()


workspaces = _Workspaces()

DEV_WAIT_TIMEOUT = 1


def device_status(device: torch.device | None = None) -> int:
    """Synchronise the device's current stream and return (and clear) the
    device error word: 0 none, 1 a bounded wait expired, 2 an embedding id
    out of range.  After 1 the scratch of the calls may hold stale slots: the
    library re-zeroes its own fixed array, and this re-zeroes the workspaces
    the Python layer manages for the device."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        code = load().gsq_device_status(stream_ptr(dev))
        if code < 0:
            check(code)
        if code == DEV_WAIT_TIMEOUT:
            workspaces.reset(dev)
            torch.cuda.synchronize(dev)
    return code
