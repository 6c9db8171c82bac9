"""Output-row tensor parallelism on real GPUs: two NCCL ranks, each holding
half of a packed projection's rows, must reproduce the single-GPU result
(matvec and matmul paths).  Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    from gsq_b200.parallel import RowParallelLinear
    from gsq_b200.quant.synthetic import random_matrix_torch
    from gsq_b200.runtime import PackedWeight
    from gsq_b200.runtime.kernels import quantized_matmul, quantized_matvec
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        ok = True
        for qtype, n, k in (("IQ3_S", 1024, 2048), ("Q4_K", 512, 5120)):
            packed = random_matrix_torch(qtype, n, k, seed=3, device=dev)  # same bytes on every rank
            w = PackedWeight.from_packed("w", packed, qtype, (n, k), device=dev)
            layer = RowParallelLinear(w)
            for rows in (1, 40):
                g = torch.Generator(device=dev).manual_seed(rows)
                x = torch.randn(rows, k, device=dev, dtype=torch.float16, generator=g)
                y = layer(x).float()
                if rows == 1:
                    ref = quantized_matvec(x, packed, qtype=qtype, out_features=n, in_features=k,
                                           out_dtype=torch.float32)
                else:
                    ref = quantized_matmul(x, packed, qtype=qtype, out_features=n, in_features=k,
                                           out_dtype=torch.float32)
                err = float((y - ref).norm() / ref.norm())
                ok = ok and y.shape == ref.shape and err <= 1e-3
        torch.cuda.synchronize()
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_row_parallel_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    results = sorted(q.get(timeout=5) for _ in range(2))
    assert results == [(0, True), (1, True)]
