"""Host logic of output-row tensor parallelism, on CPU with gloo ranks.

The local compute is the CPU oracle here (the CUDA kernels are covered by the
GPU tests); what is checked is the byte-range sharding of packed rows and the
rank-major all-gather that reassembles y."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gsq_b200.parallel import gather_rows, shard_bounds, shard_packed
from gsq_b200.parallel.tp import RowParallelLinear
from gsq_b200.quant.synthetic import random_activations, random_matrix
from gsq_b200.runtime import PackedWeight


def test_shard_bounds():
    assert shard_bounds(17408, 8, 7) == (15232, 17408)
    assert shard_bounds(5120, 2, 0) == (0, 2560)
    with pytest.raises(ValueError):
        shard_bounds(10, 4, 0)
    with pytest.raises(ValueError):
        shard_bounds(8, 2, 2)


@pytest.mark.parametrize("qtype", ["Q4_K", "IQ1_S", "Q6_K"])
def test_shards_concatenate_to_full(qtype):
    import oracle
    n, k = 64, 512
    packed = torch.from_numpy(random_matrix(qtype, n, k, seed=2))
    parts = [shard_packed(packed, qtype, n, k, 4, r) for r in range(4)]
    assert torch.equal(torch.cat(parts), packed)
    full = oracle.dequantize(packed.numpy(), qtype).reshape(n, k)
    lo, hi = shard_bounds(n, 4, 2)
    np.testing.assert_array_equal(oracle.dequantize(parts[2].numpy(), qtype).reshape(-1, k), full[lo:hi])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, qtype, result_q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, k = 48, 512
        packed = random_matrix(qtype, n, k, seed=9)
        w = PackedWeight.from_packed("w", packed, qtype, (n, k), device=None)
        x = torch.from_numpy(random_activations(3, k, seed=1).astype(np.float32))

        def local(xx, shard_holder=[]):
            s = shard_holder[0]
            y = oracle.matmul_c(xx.numpy(), s.data.numpy(), qtype, s.logical_shape[0], k)
            return torch.from_numpy(y.astype(np.float32))

        holder = []
        layer = RowParallelLinear(w, local_fn=lambda xx: local(xx, holder))
        holder.append(layer.shard)
        y = layer(x)
        exp = oracle.matmul_c(x.numpy(), packed, qtype, n, k)
        ok = np.allclose(y.numpy(), exp, rtol=1e-5, atol=1e-5) and y.shape == (3, n)
        # gather of rank-tagged slices keeps rank-major order
        tag = torch.full((2, 3), float(rank))
        g = gather_rows(tag)
        ok = ok and torch.equal(g[0], torch.tensor([float(r) for r in range(world) for _ in range(3)]))
        result_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_parallel_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, "IQ2_XS", q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = sorted(q.get(timeout=5) for _ in range(world))
    assert [r for r in results] == [(r, True) for r in range(world)]


def _failing_worker(rank, world, port, result_q):
    """Rank 1 fails before the step's gather; rank 0 must learn of it on the
    host, from the collective's error, within the group's short timeout."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            result_q.put((rank, "raised"))
            raise SystemExit(0)  # leaves between steps: nothing of it in flight
        t0 = time.time()
        try:
            gather_rows(torch.ones(2, 3))
            result_q.put((rank, "no error"))
        except RuntimeError:
            result_q.put((rank, "error" if time.time() - t0 < 60 else "late"))
    finally:
        if rank == 0:
            dist.destroy_process_group()


def test_peer_failure_surfaces_on_host_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    results = sorted(q.get(timeout=5) for _ in range(2))
    assert results == [(0, "error"), (1, "raised")]
