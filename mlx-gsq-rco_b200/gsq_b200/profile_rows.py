"""Matvec at 1, 2, 4 and 8 activation rows against the tiled matmul at 8 and
16 tokens, on the same packed matrices.

    python -m gsq_b200.profile_rows [QTYPE,QTYPE,...]

The matvec runs through ``gsq_qmv`` directly at every row count (the Python
``quantized_matvec`` reroutes 8 and more rows to the matmul); rows beyond
two run as two-row tiles along the grid's z axis, each streaming the whole
matrix.  Per case: a CUDA graph of 16 calls, replayed 4 times, timed with
CUDA events; prints one JSON line per matrix with microseconds per call.
"""
from __future__ import annotations

import json
import sys

import torch

from . import _lib
from .quant.layouts import type_id
from .quant.synthetic import random_matrix_torch
from .runtime.kernels import quantized_matmul

SHAPES = ((34816, 5120), (5120, 17408), (5120, 5120))


def _time(fn) -> float:
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            for _ in range(16):
                fn()
    torch.cuda.current_stream().wait_stream(st)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(4):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / 64


def _matvec(lib, tid: int, x: torch.Tensor, w: torch.Tensor, n: int, k: int):
    rows = x.shape[0]
    y = torch.empty((rows, n), dtype=torch.float32, device=x.device)
    need = lib.gsq_qmv_workspace_size(tid, n, k, rows)
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=x.device)

    def run():  # on the current stream: the capturing one inside a graph capture
        _lib.check(lib.gsq_qmv(tid, x.data_ptr(), _lib.DTYPE_CODES[x.dtype], w.data_ptr(), n, k, rows,
                               y.data_ptr(), _lib.DTYPE_CODES[torch.float32], ws.data_ptr(), need,
                               _lib.stream_ptr(x.device)))
    return run


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    types = argv[0].split(",") if argv else ["IQ2_XS", "IQ3_S", "IQ4_XS", "Q4_K", "Q6_K"]
    dev = torch.device("cuda", 0)
    lib = _lib.load()
    for q in types:
        for n, k in SHAPES:
            w = random_matrix_torch(q, n, k, seed=3, device=dev)
            out = {"type": q, "N": n, "K": k}
            for r in (1, 2, 4, 8):
                x = torch.randn(r, k, device=dev, dtype=torch.float16)
                out[f"qmv_rows{r}_us"] = round(_time(_matvec(lib, type_id(q), x, w, n, k)), 2)
            for m in (8, 16):
                x = torch.randn(m, k, device=dev, dtype=torch.float16)
                out[f"qmm_m{m}_us"] = round(_time(lambda: quantized_matmul(
                    x, w, qtype=q, out_features=n, in_features=k, out_dtype=torch.float32)), 2)
            out["device_status"] = int(lib.gsq_device_status(None))
            print(json.dumps(out), flush=True)
            del w


if __name__ == "__main__":
    main()
