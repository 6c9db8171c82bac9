"""Benchmark of the packed-GGUF hot path on B200 (driver contract).

One *step* = one pass of the batch-1 decode matvec over BASELINE config 2:
the 11 packed types x {5120->5120, 5120->17408, 17408->5120}, fp16
activations N(0,1), seeded synthetic packed weights (886 MB per step, far
larger than the 126 MB L2, so no step reuses another's weights from L2).

  value       whole-job QMV throughput in packed-weight GB/s: packed bytes of
              the sweep x steps / device time of the timed region (CUDA graph
              replays of the step, CUDA events, max over ranks).  One step is
              33 launches of the QMV kernel, nothing else.
  e2e         the same metric through the public Python API with host
              buffers: every step copies each projection's activation from
              pinned host memory and reads the result back.
  roofline    the QMV kernel inside the timed region: algorithmic bytes of a
              step (packed + 2K + 4N per call) / the step's CUDA-event time,
              vs the measured HBM copy bandwidth.
  qmv_sweep   per configuration: a CUDA graph of 24 launches over a ring of
              distinct weight copies (working set > 2x L2), CUDA events.
  qmm_prefill config 3 at M=512 (tcgen05 QMM) in TFLOP/s vs measured bf16 peak;
              on one GPU also M = 16, 182, 2048 against the max(FLOP, byte)
              roofline (``by_M``).
  model       config 4: the 27B Qwen3.5-hybrid decoder with random-init
              packed weights; prefill (182 and 512 tokens) and batch-1
              decode tok/s (CUDA-graph replay per token); with --gpus N
              (config 5) split by output rows over the N ranks.
  cpu_baseline the reference's CPU path (gguf-py dequantize, which
              mlx_gsq/quant/reference.py:10-18 calls, + numpy matvec) on a
              bounded sample of the same workload.

--gpus N (torchrun): each projection is split by output rows over the N
ranks (tensor parallel, strong scaling: total work fixed); the row gather is
fused into the kernels (the matvec sends every value to each peer's inbox
over NVLink, the matmul stores its tiles into every rank's output).
--impl reference runs the CPU reference path only (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "mlx-gsq-rco_b200"))

TYPES = ("IQ1_M", "IQ1_S", "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ4_XS", "Q2_K", "Q4_K", "Q6_K")
SHAPES = ((5120, 5120), (17408, 5120), (5120, 17408))  # (N out, K in)
QMM_TYPES = ("IQ2_XS", "IQ3_S", "IQ4_XS", "Q6_K")
QMM_SHAPES = ((17408, 5120), (5120, 17408))
METRIC = "decode tok/s (batch 1) + QMV packed-byte HBM GB/s vs peak; prefill tok/s at M=512"
BLOCK_BYTES = {"IQ1_M": 56, "IQ1_S": 50, "IQ2_XXS": 66, "IQ2_XS": 74, "IQ2_S": 82, "IQ3_XXS": 98, "IQ3_S": 110,
               "IQ4_XS": 136, "Q2_K": 84, "Q4_K": 144, "Q6_K": 210}


def packed_bytes(q, n, k):
    return n * (k // 256) * BLOCK_BYTES[q]


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return {"hbm": p["hbm_gbs"], "bf16": p["bf16_tflops"], "src": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "25",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0:  # sampling has started before timing does
                time.sleep(0.01)
            self.lines.clear()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_reference_sample(time_budget_s: float = 20.0):
    """The reference's CPU path: gguf-py dequantize (what dequantize_reference
    calls) + numpy fp32 matvec, on 5120x5120 matrices of the sweep's types,
    until the time budget is spent.  Returns packed-byte GB/s and the sample."""
    import gguf
    from gsq_b200.quant.synthetic import random_activations, random_matrix
    done_bytes, spent, sample = 0, 0.0, []
    for q in ("Q4_K", "IQ2_XS", "IQ3_S", "Q6_K", "IQ4_XS", "IQ1_S"):
        n = k = 5120
        packed = random_matrix(q, n, k, seed=0)
        x = random_activations(1, k, seed=0).astype(np.float32)
        t0 = time.perf_counter()
        deq = gguf.dequantize(packed.reshape(-1, BLOCK_BYTES[q]), gguf.GGMLQuantizationType[q]).reshape(n, k)
        _ = x @ deq.T
        dt = time.perf_counter() - t0
        done_bytes += packed.size
        spent += dt
        sample.append(f"{q} {n}x{k}")
        if spent > time_budget_s:
            break
    return done_bytes / spent / 1e9, spent, sample


def run_reference(args, rank):
    if rank != 0:
        return
    gbs, spent, sample = cpu_reference_sample(args.cpu_budget)
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s (packed weight bytes, QMV batch 1)",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config-2 QMV sweep, bounded CPU sample: " + ", ".join(sample),
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "reference",
                         "sample": f"gguf-py 0.19.0 dequantize + numpy matvec over {', '.join(sample)} "
                                   f"({spent:.1f} s)"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def decode_tok_s(per):
    """Batch-1 decode tokens/s of one FFN-shaped projection pair per type
    (17408x5120 up + 5120x17408 down), from the per-configuration timings:
    1 / (t_up + t_down).  A per-pair figure, not a model's tok/s."""
    out = {}
    for q in TYPES:
        t = [r["us"] for r in per if r["type"] == q and (r["N"], r["K"]) in ((17408, 5120), (5120, 17408))]
        if len(t) == 2:
            out[q] = round(1e6 / sum(t), 1)
    return out or None


def qmm_by_m(dev, pk, ms=(16, 182, 2048)):
    """Config 3 at the other token counts, one GPU: for each M, one CUDA graph
    runs the 8 projections (4 types x 2 shapes, 369 MB of distinct packed
    weights, > 2x L2) back to back; replayed, CUDA events.  Reported against
    the max(FLOP, byte) roofline: bound = max(2MNK / bf16 peak, bytes / HBM
    peak) summed over the 8 projections, bytes = packed + 2MK (bf16 x) +
    4MN (fp32 y)."""
    import torch
    from gsq_b200.quant.synthetic import random_matrix_torch
    from gsq_b200.runtime.kernels import quantized_matmul

    mats = [(q, n, k, random_matrix_torch(q, n, k, seed=7, device=dev)) for q in QMM_TYPES for (n, k) in QMM_SHAPES]
    out = []
    for m in ms:
        xs = {k: torch.randn(m, k, device=dev, dtype=torch.bfloat16,
                             generator=torch.Generator(device=dev).manual_seed(11)) for k in {5120, 17408}}

        def run():
            for q, n, k, w in mats:
                quantized_matmul(xs[k], w, qtype=q, out_features=n, in_features=k, out_dtype=torch.float32)

        for _ in range(3):
            run()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream(device=dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                for _ in range(2):
                    run()
        torch.cuda.current_stream(dev).wait_stream(st)
        g.replay()
        torch.cuda.synchronize()
        reps = 4
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / (2 * reps)  # seconds per pass over the 8 projections
        del g
        flops = sum(2.0 * m * n * k for _, n, k, _ in mats)
        nbytes = sum(packed_bytes(q, n, k) + 2 * m * k + 4 * m * n for q, n, k, _ in mats)
        bound = sum(max(2.0 * m * n * k / (pk["bf16"] * 1e12), (packed_bytes(q, n, k) + 2 * m * k + 4 * m * n)
                        / (pk["hbm"] * 1e9)) for q, n, k, _ in mats)
        out.append({"M": m, "us_per_pass": round(t * 1e6, 1), "tflops": round(flops / t / 1e12, 1),
                    "gbs": round(nbytes / t / 1e9, 1), "roofline_frac": round(bound / t, 4),
                    "bound": "hbm" if nbytes / (pk["hbm"] * 1e9) > flops / (pk["bf16"] * 1e12) else "tensor"})
        del xs
    del mats
    torch.cuda.empty_cache()
    return out


def model_bench(dev, pk, world=1, prompt=182, decode_tokens=64, prefill_m=512):
    """Config 4 (BASELINE): the Qwen3.5-hybrid 27B decoder (64 layers) with
    random-init packed weights of the config's type mix.  A ``prompt``-token
    prefill, then ``decode_tokens`` greedy decode tokens at batch 1, each a
    replay of the captured decode-step graph (embedding -> 64 layers -> LM
    head -> argmax); and a ``prefill_m``-token prefill.  CUDA events around
    each timed region; every decode token reads all packed projections
    (12 GB, ~90x L2).  With ``world`` > 1 (config 5) every packed projection
    is split by output rows over the ranks (the gathers fused into the matvec
    and the matmul epilogue); times are the max over ranks."""
    import torch
    import torch.distributed as dist
    from gsq_b200.models import Qwen35Config, build_qwen35, random_weights

    cfg = Qwen35Config()
    w = random_weights(cfg, dev, seed=0)  # the same bytes on every rank; each keeps its rows
    model = build_qwen35(w, cfg, dev, max_len=prefill_m + decode_tokens + 16,
                         group=dist.group.WORLD if world > 1 else None)
    del w
    torch.cuda.empty_cache()
    gen = torch.Generator(device=dev).manual_seed(1)

    def max_over_ranks(t):
        if world > 1:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    def timed(fn, reps):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / 1e3 / reps)

    out = {"workload": "config 4: Qwen3.5-hybrid 27B (64 layers, 48 gated-DeltaNet + 16 GQA), random-init packed "
                       "weights (embedding/LM head Q6_K, FFN gate/up IQ2_XS|IQ2_S, down Q4_K, attention IQ3_S|IQ4_XS)",
           "packed_bytes_per_token": model.packed_bytes_per_token()}
    for T in (prompt, prefill_m):
        ids = torch.randint(0, cfg.vocab_size, (T,), device=dev, generator=gen, dtype=torch.int32)
        model.prefill(ids)  # warm-up (workspaces, cuBLAS / attention plans)
        torch.cuda.synchronize()
        t = timed(lambda: model.prefill(ids), 3)
        out[f"prefill_{T}_ms"] = round(t * 1e3, 2)
        out[f"prefill_{T}_tok_s"] = round(T / t, 1)

    ids = torch.randint(0, cfg.vocab_size, (prompt,), device=dev, generator=gen, dtype=torch.int32)
    model.prefill(ids)
    model.decode_step()
    model.capture_decode()
    model.replay_decode(3)  # warm-up replays
    t = timed(lambda: model.replay_decode(decode_tokens), 1) / decode_tokens
    gbs = out["packed_bytes_per_token"] / t / 1e9
    out.update({"decode_tokens": decode_tokens, "decode_ms_per_token": round(t * 1e3, 3),
                "decode_tok_s": round(1.0 / t, 1), "decode_packed_gbs": round(gbs, 1),
                "decode_roofline_frac": round(gbs / pk["hbm"], 4),
                "decode_note": "batch 1 after the prompt prefill; each token one CUDA-graph replay of the whole "
                               "step; roofline = packed weight bytes per token / time vs measured HBM copy peak"
                               + (f" x {world} GPUs" if world > 1 else "")})
    if world > 1:
        out["decode_roofline_frac"] = round(gbs / (pk["hbm"] * world), 4)
        out["parallelism"] = (f"tp{world}: every packed projection split by output rows; the row gathers fused "
                              "into the matvec (decode) and the matmul epilogue (prefill) over NVLink")
    model.close()
    del model
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-qmm", action="store_true")
    ap.add_argument("--no-model", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist
    from gsq_b200 import _lib
    from gsq_b200.quant.synthetic import random_matrix_torch
    from gsq_b200.runtime.kernels import quantized_matmul, quantized_matvec

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        from gsq_b200.parallel import GatherRegion, quantized_matmul_gather, quantized_matvec_gather
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    pk = peaks()

    # ---- workload: every rank holds its row shard of every projection ----
    cfgs = []
    for ti, q in enumerate(TYPES):
        for si, (n, k) in enumerate(SHAPES):
            full = random_matrix_torch(q, n, k, seed=100 * ti + si, device=dev)
            rows = n // world
            rb = (k // 256) * BLOCK_BYTES[q]
            shard = full[rank * rows * rb:(rank + 1) * rows * rb].clone()
            del full
            x = torch.randn(1, k, device=dev, dtype=torch.float16, generator=torch.Generator(device=dev).manual_seed(ti))
            # Ranks > 1: the gathered output of every configuration lives in
            # its own region (the gather is fused into the matvec kernel).
            region = GatherRegion(1, n) if world > 1 else None
            cfgs.append(dict(q=q, n=n, k=k, rows=rows, packed=shard, x=x, region=region,
                             bytes=packed_bytes(q, n, k), alg=packed_bytes(q, rows, k) + 2 * k + 4 * rows))
    step_bytes = sum(c["bytes"] for c in cfgs)
    torch.cuda.synchronize()

    def matvec(c, x):
        """One projection: y, or (ranks > 1) every rank's rows gathered in c's region."""
        if world > 1:
            return quantized_matvec_gather(x, c["packed"], qtype=c["q"], out_features=c["rows"], in_features=c["k"],
                                           region=c["region"], row0=rank * c["rows"])
        return quantized_matvec(x, c["packed"], qtype=c["q"], out_features=c["rows"], in_features=c["k"],
                                out_dtype=torch.float32)

    def step():
        for c in cfgs:
            matvec(c, c["x"])

    # warm up eagerly (allocates workspaces, sets kernel attributes), then capture
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap_stream = torch.cuda.Stream(device=dev)
    cap_stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(cap_stream):
        with torch.cuda.graph(graph, stream=cap_stream):
            step()
    torch.cuda.current_stream(dev).wait_stream(cap_stream)
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_per_step = ms / args.steps
    value = step_bytes * args.steps / (ms / 1e3) / 1e9

    # ---- roofline of the QMV kernel over the timed region ----
    alg_step = sum(c["alg"] for c in cfgs)
    achieved = alg_step / (ms_per_step / 1e3) / 1e9
    traffic = None
    tpath = os.path.join(REPO, "profiles", "qmv_traffic.json")
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath)).get("dram_bytes_per_launch")
        except (OSError, ValueError):
            traffic = None
    roofline = {"bound": "hbm", "kernel": "gsq::qmv_kernel", "achieved": round(achieved, 1), "peak": pk["hbm"],
                "unit": "GB/s", "frac": round(achieved / pk["hbm"], 4), "peak_source": pk["src"] + " (copy bandwidth)",
                "traffic": traffic,
                "achieved_definition": "algorithmic bytes of one step (33 launches: packed + 2K + 4N each) / "
                                       "CUDA-event time of one step in the timed region"}

    # ---- per configuration: graph of 24 launches over a ring of copies ----
    per = []
    if world == 1:
        l2 = 126 << 20
        for c in cfgs:
            nbytes = c["packed"].numel()
            ncopy = max(8, min(24, -(-2 * l2 // nbytes)))
            ring = [c["packed"]] + [c["packed"].clone() for _ in range(ncopy - 1)]
            reps = 24
            for i in range(2):
                quantized_matvec(c["x"], ring[i % ncopy], qtype=c["q"], out_features=c["rows"], in_features=c["k"],
                                 out_dtype=torch.float32)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            st = torch.cuda.Stream(device=dev)
            st.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(st):
                with torch.cuda.graph(g, stream=st):
                    for i in range(reps):
                        quantized_matvec(c["x"], ring[i % ncopy], qtype=c["q"], out_features=c["rows"],
                                         in_features=c["k"], out_dtype=torch.float32)
            torch.cuda.current_stream(dev).wait_stream(st)
            for _ in range(2):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
            t_us = e0.elapsed_time(e1) * 1e3 / (5 * reps)
            per.append({"type": c["q"], "N": c["n"], "K": c["k"], "us": round(t_us, 2),
                        "GBs": round(c["alg"] / (t_us / 1e6) / 1e9, 1),
                        "frac": round(c["alg"] / (t_us / 1e6) / 1e9 / pk["hbm"], 3)})
            del g, ring
            torch.cuda.empty_cache()

    # ---- e2e through the C ABI with host buffers ----
    if world == 1:
        # As a C-ABI host drives it: the step's activations sit in one pinned
        # host buffer and go to the device in one copy; one gsq_qmv call per
        # projection (device pointers prepared once); the outputs come back
        # to one pinned host buffer in one copy; one synchronisation per step.
        from gsq_b200.quant.layouts import type_id
        lib = _lib.load()
        xoff, yoff = [], []
        nx = ny = 0
        for c in cfgs:
            xoff.append(nx)
            yoff.append(ny)
            nx += -(-c["k"] // 8) * 8  # keep every activation row 16-byte aligned
            ny += c["rows"]
        host_xb = torch.zeros(nx, dtype=torch.float16).pin_memory()
        for c, o in zip(cfgs, xoff):
            host_xb[o:o + c["k"]] = c["x"].reshape(-1).cpu()
        host_yb = torch.empty(ny, dtype=torch.float32).pin_memory()
        dev_xb = torch.empty(nx, dtype=torch.float16, device=dev)
        dev_yb = torch.empty(ny, dtype=torch.float32, device=dev)
        need = max(lib.gsq_qmv_workspace_size(type_id(c["q"]), c["rows"], c["k"], 1) for c in cfgs)
        ws = _lib.workspaces.get(dev, need, "qmv")
        wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
        stream = _lib.stream_ptr(dev)
        calls = [(type_id(c["q"]), dev_xb.data_ptr() + 2 * xo, _lib.DTYPE_CODES[torch.float16], c["packed"].data_ptr(),
                  c["rows"], c["k"], 1, dev_yb.data_ptr() + 4 * yo, _lib.DTYPE_CODES[torch.float32], wsp, wsn, stream)
                 for c, xo, yo in zip(cfgs, xoff, yoff)]
        h2d, d2h = nx * 2, ny * 4
        qmv = lib.gsq_qmv

        def e2e_step():
            dev_xb.copy_(host_xb, non_blocking=True)
            for args_ in calls:
                rc = qmv(*args_)
                if rc:
                    _lib.check(rc)
            host_yb.copy_(dev_yb, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
        e2e_path = ("activations of the step in one pinned host buffer -> one copy to the device -> one gsq_qmv "
                    "C-ABI call per projection (ctypes, device pointers prepared once) -> outputs in one copy to "
                    "pinned host memory; one stream synchronisation per step")
    else:
        # The same with the gather fused in: one gsq_qmv_gather call per
        # projection (this rank's rows; every rank's rows land in the
        # projection's gather region), then each region's gathered row is
        # copied to the one pinned host buffer.
        from gsq_b200.quant.layouts import type_id
        lib = _lib.load()
        xoff, yoff = [], []
        nx = ny = 0
        for c in cfgs:
            xoff.append(nx)
            yoff.append(ny)
            nx += -(-c["k"] // 8) * 8
            ny += c["n"]
        host_xb = torch.zeros(nx, dtype=torch.float16).pin_memory()
        for c, o in zip(cfgs, xoff):
            host_xb[o:o + c["k"]] = c["x"].reshape(-1).cpu()
        host_yb = torch.empty(ny, dtype=torch.float32).pin_memory()
        dev_xb = torch.empty(nx, dtype=torch.float16, device=dev)
        need = max(lib.gsq_qmv_workspace_size(type_id(c["q"]), c["rows"], c["k"], 1) for c in cfgs)
        ws = _lib.workspaces.get(dev, need, "qmv")
        wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
        stream = _lib.stream_ptr(dev)
        calls = [(type_id(c["q"]), dev_xb.data_ptr() + 2 * xo, _lib.DTYPE_CODES[torch.float16], c["packed"].data_ptr(),
                  c["rows"], c["k"], 1, c["region"].regions, world, rank, rank * c["rows"], c["n"], wsp, wsn, stream)
                 for c, xo in zip(cfgs, xoff)]
        outs = [(host_yb[yo:yo + c["n"]], c["region"].y.reshape(-1)) for c, yo in zip(cfgs, yoff)]
        h2d, d2h = nx * 2, ny * 4
        qmvg = lib.gsq_qmv_gather

        def e2e_step():
            dev_xb.copy_(host_xb, non_blocking=True)
            for args_ in calls:
                rc = qmvg(*args_)
                if rc:
                    _lib.check(rc)
            for hy, y in outs:
                hy.copy_(y, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
        e2e_path = ("activations of the step in one pinned host buffer -> one copy to the device -> one "
                    "gsq_qmv_gather C-ABI call per projection (this rank's rows, every rank's rows gathered) -> "
                    "each gathered output copied to one pinned host buffer; one stream synchronisation per step")

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_steps = max(3, args.steps // 4)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(e2e_steps):
        e2e_step()
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = t0.elapsed_time(t1)
    # the host copy of the outputs is the library's result
    ref = matvec(cfgs[0], cfgs[0]["x"]).reshape(-1).cpu()
    if not torch.allclose(host_yb[:ref.numel()], ref, rtol=1e-6, atol=0):
        raise RuntimeError("end-to-end outputs differ from the library call")
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": round(step_bytes * e2e_steps / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "path": e2e_path}

    # ---- QMM prefill, config 3 at M=512 (ranks > 1: each rank's row shard,
    # with the gather fused into the matmul's epilogue) ----
    qmm = None
    if not args.no_qmm:
        qres = []
        flops_total, t_qmm = 0.0, 0.0
        for q in QMM_TYPES:
            for (n, k) in QMM_SHAPES:
                rows = n // world
                full = random_matrix_torch(q, n, k, seed=7, device=dev)
                rb = (k // 256) * BLOCK_BYTES[q]
                w = full[rank * rows * rb:(rank + 1) * rows * rb].clone()
                del full
                x = torch.randn(512, k, device=dev, dtype=torch.bfloat16,
                                generator=torch.Generator(device=dev).manual_seed(11))
                region = GatherRegion(512, n) if world > 1 else None

                def prefill():
                    if world > 1:
                        quantized_matmul_gather(x, w, qtype=q, out_features=rows, in_features=k, region=region,
                                                row0=rank * rows)
                    else:
                        quantized_matmul(x, w, qtype=q, out_features=rows, in_features=k, out_dtype=torch.float32)

                for _ in range(2):
                    prefill()
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                st = torch.cuda.Stream(device=dev)
                st.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(st):
                    with torch.cuda.graph(g, stream=st):
                        for _ in range(8):
                            prefill()
                torch.cuda.current_stream(dev).wait_stream(st)
                g.replay()
                torch.cuda.synchronize()
                if world > 1:
                    dist.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(3):
                    g.replay()
                e1.record()
                torch.cuda.synchronize()
                t_ms = e0.elapsed_time(e1) / 24
                if world > 1:
                    tt = torch.tensor([t_ms], device=dev)
                    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                    t_ms = float(tt.item())
                    region.close()
                del g
                fl = 2.0 * 512 * n * k
                flops_total += fl
                t_qmm += t_ms / 1e3
                qres.append({"type": q, "N": n, "K": k, "us": round(t_ms * 1e3, 1),
                             "TFLOPs": round(fl / (t_ms / 1e3) / 1e12, 1)})
                del w
        tf = flops_total / t_qmm / 1e12
        qmm = {"M": 512, "tflops": round(tf, 1), "peak": round(pk["bf16"] * world, 1),
               "frac": round(tf / (pk["bf16"] * world), 4),
               "prefill_tok_s_per_projection_pair": {
                   q: round(512.0 / sum(r["us"] * 1e-6 for r in qres if r["type"] == q), 1) for q in QMM_TYPES},
               "per_shape": qres,
               "note": "includes the bf16->fp16 activation pre-pass; weights decoded once per 128x128 tile; "
                       "CUDA graph of 8 launches, CUDA events" + (
                           f"; {world} ranks: row shards, the gather fused into the matmul epilogue, max over ranks, "
                           f"peak = {world} x the measured bf16 peak" if world > 1 else "")}

    if qmm is not None and world == 1:
        qmm["by_M"] = qmm_by_m(dev, pk)
    model = None
    if not args.no_model:
        try:
            model = model_bench(dev, pk, world)
        except Exception as e:  # recorded in the line; the QMV and QMM results above still stand
            model = {"error": f"{type(e).__name__}: {e}"[:300]}

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        gbs, spent, sample = cpu_reference_sample(args.cpu_budget)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": os.cpu_count(), "kind": "reference",
               "sample": f"gguf-py 0.19.0 dequantize + numpy matvec over {', '.join(sample)} ({spent:.1f} s)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s (packed weight bytes, QMV batch 1)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8",
            "dtype_note": "decoded packed entries (s8/u8) x two int8 activation levels on the tensor cores, "
                          "s32 accumulate, fp32 scales and output; fp16 activations in",
            "data": "synthetic",
            "config": {"workload": "config-2 QMV sweep: 11 types x {5120->5120, 5120->17408, 17408->5120}, batch 1",
                       "bytes_per_step": step_bytes, "l2": "inputs larger than L2 (886 MB per step)",
                       "parallelism": (f"tp{world} (output rows; the gather is fused into the matvec: each "
                                       f"value goes to every rank's inbox over NVLink)") if world > 1 else "single GPU",
                       "timing": "CUDA graph of one step, replayed; CUDA events"},
            "roofline": roofline, "qmv_sweep": per, "qmm_prefill": qmm, "cpu_baseline": cpu, "e2e": e2e,
            "decode_tok_s_per_projection_pair": decode_tok_s(per), "model": model,
            "clocks": clocks.summary(), "gpu_launches": args.steps * len(cfgs),
        }
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        for c in cfgs:
            c["region"].close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
