"""Output-row tensor parallelism on real GPUs: 2, 4 or 8 NCCL ranks, each
holding its slice of a packed projection's rows, must reproduce the
single-GPU result (matvec with the gather fused in, matmul with the gather
fused into its epilogue, and the NCCL all-gather path), also over repeated
calls and CUDA-graph replays of the fused gather.  A projection split by
input blocks (partials all-reduced) must reproduce the whole product.  The
model harness runs both split by output rows and in the head-split layout,
against the same model on one GPU.  Each world size is skipped when fewer
GPUs are visible."""
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
    fails = []

    def check(label, a, b, tol=1e-3):
        e = float((a.float() - b.float()).norm() / b.float().norm())
        if not (a.shape == b.shape and e <= tol):
            fails.append(f"{label}: {e:.3g}")
        return True

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
                check(f"RowParallelLinear {qtype} rows {rows}", y, ref)
        # Matvec with the gather fused in: against the NCCL path and one GPU,
        # repeated on two alternating regions (flag counts advance per call),
        # then replayed from a CUDA graph.
        from gsq_b200 import _lib
        from gsq_b200.parallel import GatherRegion, quantized_matvec_gather, shard_packed
        n, k = 2048, 5120
        packed = random_matrix_torch("IQ2_XS", n, k, seed=5, device=dev)
        shard = shard_packed(packed, "IQ2_XS", n, k, world, rank)
        regions = [GatherRegion(1, n) for _ in range(2)]
        xs = [torch.randn(1, k, device=dev, dtype=torch.float16, generator=torch.Generator(device=dev).manual_seed(i))
              for i in range(2)]
        refs = [quantized_matvec(x, packed, qtype="IQ2_XS", out_features=n, in_features=k, out_dtype=torch.float32)
                for x in xs]
        for it in range(20):
            i = it % 2
            y = quantized_matvec_gather(xs[i], shard, qtype="IQ2_XS", out_features=n // world, in_features=k,
                                        region=regions[i], row0=rank * (n // world))
            check(f"matvec gather call {it}", y, refs[i])
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream(device=dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                for i in range(2):
                    quantized_matvec_gather(xs[i], shard, qtype="IQ2_XS", out_features=n // world, in_features=k,
                                            region=regions[i], row0=rank * (n // world))
        torch.cuda.current_stream(dev).wait_stream(st)
        for _ in range(5):
            regions[0].y.zero_()
            regions[1].y.zero_()
            torch.cuda.synchronize()
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            for i in range(2):
                check(f"matvec gather graph {i}", regions[i].y, refs[i])
        # Tiled matmul with the gather fused into its epilogue (split-K and
        # whole-K shapes), repeated on one region.
        from gsq_b200.parallel import quantized_matmul_gather
        # Both ways of delivering the tiles: one multicast store per value
        # through the NVSwitch (symmetric-memory regions, where the GPUs
        # offer it) and one store per rank over NVLink.
        # fp16 regions too (16-byte pieces of 8 rows; 1000 rows: shards whose
        # first row is not a multiple of 8 take the per-value path).
        for multicast in (True, False):
            for qtype, n2, k2, ydt in (("IQ4_XS", 2048, 5120, torch.float32), ("IQ4_XS", 2048, 5120, torch.float16),
                                       ("Q6_K", 1024, 17408, torch.float32), ("Q6_K", 1024, 17408, torch.float16),
                                       ("Q4_K", 1000, 2048, torch.float16)):
                packed2 = random_matrix_torch(qtype, n2, k2, seed=6, device=dev)
                shard2 = shard_packed(packed2, qtype, n2, k2, world, rank)
                region2 = GatherRegion(64, n2, multicast=multicast, dtype=ydt)
                if not multicast and region2.mc is not None:
                    fails.append("multicast region without asking")
                for it in range(3):
                    x2 = torch.randn(64, k2, device=dev, dtype=torch.bfloat16,
                                     generator=torch.Generator(device=dev).manual_seed(10 + it))
                    ref2 = quantized_matmul(x2, packed2, qtype=qtype, out_features=n2, in_features=k2,
                                            out_dtype=torch.float32)
                    y2 = quantized_matmul_gather(x2, shard2, qtype=qtype, out_features=n2 // world, in_features=k2,
                                                 region=region2, row0=rank * (n2 // world))
                    if y2.dtype != ydt:
                        fails.append(f"region dtype {y2.dtype}")
                    check(f"matmul gather mc={multicast} {qtype} {ydt} N={n2} it {it}", y2, ref2)
                    # The next call on this region stores into every rank's copy: no rank
                    # may start it before every rank has read this call's rows.
                    dist.barrier()
                region2.close()
            # A 2048-token call whose shard has more tiles than SMs (2 ranks:
            # 5120 rows x 4 token groups = 160 tiles): full waves, then the last
            # wave's tiles with K split, each launch gathering its tiles.
            if world == 2:
                n4, k4 = 10240, 512
                packed4 = random_matrix_torch("IQ4_XS", n4, k4, seed=9, device=dev)
                shard4 = shard_packed(packed4, "IQ4_XS", n4, k4, world, rank)
                region4 = GatherRegion(2048, n4, multicast=multicast, dtype=torch.float16)
                x4 = torch.randn(2048, k4, device=dev, dtype=torch.bfloat16,
                                 generator=torch.Generator(device=dev).manual_seed(30))
                ref4 = quantized_matmul(x4, packed4, qtype="IQ4_XS", out_features=n4, in_features=k4,
                                        out_dtype=torch.float32)
                y4 = quantized_matmul_gather(x4, shard4, qtype="IQ4_XS", out_features=n4 // world, in_features=k4,
                                             region=region4, row0=rank * (n4 // world))
                check(f"last-wave split mc={multicast}", y4, ref4)
                dist.barrier()
                region4.close()
            # One region shared by calls of different token counts (one and
            # several 512-token groups, as a model's prefill region sees).
            n3, k3 = 1024, 5120
            packed3 = random_matrix_torch("IQ3_S", n3, k3, seed=8, device=dev)
            shard3 = shard_packed(packed3, "IQ3_S", n3, k3, world, rank)
            region3 = GatherRegion(1300, n3, multicast=multicast)
            for it, m3 in enumerate((64, 1300, 182, 600, 64)):
                x3 = torch.randn(m3, k3, device=dev, dtype=torch.bfloat16,
                                 generator=torch.Generator(device=dev).manual_seed(20 + it))
                ref3 = quantized_matmul(x3, packed3, qtype="IQ3_S", out_features=n3, in_features=k3,
                                        out_dtype=torch.float32)
                y3 = quantized_matmul_gather(x3, shard3, qtype="IQ3_S", out_features=n3 // world, in_features=k3,
                                             region=region3, row0=rank * (n3 // world))
                check(f"shared region mc={multicast} M={m3}", y3, ref3)
                dist.barrier()
            region3.close()
        status = _lib.load().gsq_device_status(None)
        if status:
            fails.append(f"device status {status}")
        del g
        for r in regions:
            r.close()
        layer.close()
        torch.cuda.synchronize()
        q.put((rank, not fails, fails))
    finally:
        dist.destroy_process_group()


def _spawn(target, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = sorted(q.get(timeout=5) for _ in range(world))
    assert [r[:2] for r in results] == [(r, True) for r in range(world)], results


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_parallel(world):
    _spawn(_worker, world)


def _input_parallel_worker(rank, world, port, q):
    """InputParallelLinear: each rank's input blocks (an uneven run, and a
    head plan's scattered blocks) with the partials all-reduced, against the
    whole matrix on one GPU (matvec and matmul paths)."""
    import torch.distributed as dist
    from datetime import timedelta
    from gsq_b200.parallel import InputParallelLinear, linear_attention_heads
    from gsq_b200.quant.synthetic import random_matrix_torch
    from gsq_b200.runtime import PackedWeight
    from gsq_b200.runtime.kernels import quantized_matvec
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    fails = []
    try:
        # ffn_down-like (uneven block runs) and ssm_out-like (a head plan's blocks)
        cases = (("Q4_K", 640, 17 * 256, None),
                 ("IQ4_XS", 512, 48 * 128, linear_attention_heads(16, 48, world, rank).out_blocks(128)))
        for qtype, n, k, blocks in cases:
            packed = random_matrix_torch(qtype, n, k, seed=4, device=dev)  # same bytes on every rank
            w = PackedWeight.from_packed("w", packed, qtype, (n, k), device=dev)
            layer = InputParallelLinear(w, blocks=blocks)
            for rows in (1, 3, 40):
                g = torch.Generator(device=dev).manual_seed(rows)
                x = torch.randn(rows, k, device=dev, dtype=torch.float16, generator=g)
                y = layer(layer.local_columns(x), out_dtype=torch.float32)
                ref = quantized_matvec(x, packed, qtype=qtype, out_features=n, in_features=k,
                                       out_dtype=torch.float32)
                e = float((y - ref).norm() / ref.norm())
                if not (y.shape == ref.shape and e <= 1e-3):
                    fails.append(f"{qtype} rows {rows}: {e:.3g}")
        q.put((rank, not fails, fails))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_input_parallel(world):
    _spawn(_input_parallel_worker, world)


def _model_worker(rank, world, port, q):
    """The Qwen3.5-hybrid harness split over the ranks against the same model
    on one GPU (same weights, built on every rank from the same seed)."""
    import torch.distributed as dist
    from datetime import timedelta
    from gsq_b200 import _lib
    from gsq_b200.models import Qwen35Config, build_qwen35, random_weights
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        cfg = Qwen35Config(hidden_size=512, intermediate_size=768, num_hidden_layers=4, num_attention_heads=4,
                           num_key_value_heads=2, vocab_size=512, linear_num_value_heads=4,
                           linear_num_key_heads=2)
        w = random_weights(cfg, dev, seed=3)
        one = build_qwen35(w, cfg, dev, max_len=64)
        tp = build_qwen35(w, cfg, dev, max_len=64, group=dist.group.WORLD)

        fails = []

        def check(label, a, b, tol=1e-3):
            """Every check runs on every rank (the calls inside are collective)."""
            e = float((a.float() - b.float()).norm() / b.float().norm())
            if not e <= tol:
                fails.append(f"{label}: {e:.3g}")

        prompt = (torch.arange(12, dtype=torch.int32, device=dev) * 41) % cfg.vocab_size
        check("prefill 12", tp.prefill(prompt), one.prefill(prompt))  # matmul, gather in the epilogue
        long_prompt = (torch.arange(40, dtype=torch.int32, device=dev) * 17) % cfg.vocab_size
        check("prefill 40", tp.prefill(long_prompt), one.prefill(long_prompt))  # the same regions, more tokens
        check("prefill 12 again", tp.prefill(prompt), one.prefill(prompt))
        for t in (5, 77, 300):  # eager decode: the fused-gather matvec
            check(f"decode {t}", tp.decode_step(t), one.decode_step(t))
        tp.capture_decode()
        one.capture_decode()
        for i in range(3):  # graph decode, greedy: both must follow the same tokens
            tp.replay_decode(1)
            one.replay_decode(1)
            check(f"graph step {i}", tp.graph_logits, one.graph_logits)
            if int(tp.cur_id.item()) != int(one.cur_id.item()):
                fails.append(f"graph step {i}: tokens differ")
        # batched decode (9 sequences: the projections run the matmul with
        # the gather fused into its epilogue; the LM head an NCCL all-gather)
        tp.release_graph()
        one.release_graph()
        tpb = build_qwen35(w, cfg, dev, max_len=64, max_batch=9, group=dist.group.WORLD)
        oneb = build_qwen35(w, cfg, dev, max_len=64, max_batch=9)
        toks = [(13 * b + 3) % cfg.vocab_size for b in range(9)]
        for m in (tpb, oneb):
            m.prefill(prompt)
            m.fork(9)
        check("batched decode 1", tpb.decode_step(toks), oneb.decode_step(toks))
        check("batched decode 2", tpb.decode_step(toks), oneb.decode_step(toks))
        torch.cuda.synchronize()
        status = _lib.load().gsq_device_status(None)
        if status:
            fails.append(f"device status {status}")
        tpb.close()
        tp.close()
        q.put((rank, not fails, fails))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_model_tensor_parallel(world):
    _spawn(_model_worker, world)


def _model_heads_worker(rank, world, port, q):
    """The harness in the head-split layout (each rank its heads and FFN
    blocks, the blocks' partial outputs all-reduced) against the same model
    on one GPU."""
    import torch.distributed as dist
    from datetime import timedelta
    from gsq_b200 import _lib
    from gsq_b200.models import Qwen35Config, build_qwen35, build_qwen35_head_split, random_weights
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        # 16 key heads: two per rank at 8 ranks (whole 256-wide blocks of
        # ssm_out); 18 FFN blocks: uneven over 4 and 8 ranks, at least 2 each
        cfg = Qwen35Config(hidden_size=512, intermediate_size=4608, num_hidden_layers=4, num_attention_heads=8,
                           num_key_value_heads=2, vocab_size=512, linear_num_value_heads=48,
                           linear_num_key_heads=16)
        w = random_weights(cfg, dev, seed=5)
        one = build_qwen35(w, cfg, dev, max_len=64, max_batch=9)
        hs = build_qwen35_head_split(w, cfg, dev, max_len=64, max_batch=9, group=dist.group.WORLD)
        fails = []

        def check(label, a, b, tol=1e-3):
            e = float((a.float() - b.float()).norm() / b.float().norm())
            if not e <= tol:
                fails.append(f"{label}: {e:.3g}")

        prompt = (torch.arange(12, dtype=torch.int32, device=dev) * 41) % cfg.vocab_size
        check("prefill 12", hs.prefill(prompt), one.prefill(prompt))
        long_prompt = (torch.arange(40, dtype=torch.int32, device=dev) * 17) % cfg.vocab_size
        check("prefill 40", hs.prefill(long_prompt), one.prefill(long_prompt))
        for t in (5, 77, 300):
            check(f"decode {t}", hs.decode_step(t), one.decode_step(t))
        hs.capture_decode()
        one.capture_decode()
        for i in range(3):
            hs.replay_decode(1)
            one.replay_decode(1)
            check(f"graph step {i}", hs.graph_logits, one.graph_logits)
            if int(hs.cur_id[0].item()) != int(one.cur_id[0].item()):
                fails.append(f"graph step {i}: tokens differ")
        hs.release_graph()
        one.release_graph()
        toks = [(13 * b + 3) % cfg.vocab_size for b in range(9)]
        for m in (hs, one):
            m.prefill(prompt)
            m.fork(9)
        check("batched decode 1", hs.decode_step(toks), one.decode_step(toks))
        check("batched decode 2", hs.decode_step(toks), one.decode_step(toks))
        torch.cuda.synchronize()
        status = _lib.load().gsq_device_status(None)
        if status:
            fails.append(f"device status {status}")
        hs.close()
        q.put((rank, not fails, fails))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_model_head_split(world):
    _spawn(_model_heads_worker, world)
