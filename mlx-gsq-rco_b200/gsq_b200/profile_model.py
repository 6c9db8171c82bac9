"""Per-kernel device time of one decode token of the Qwen3.5-hybrid harness.

    python -m gsq_b200.profile_model [prompt_tokens] [tokens]
    python -m gsq_b200.profile_model prefill [prompt_tokens]
    python -m gsq_b200.profile_model gdn
    python -m gsq_b200.profile_model batch [B] [prompt_tokens] [steps]

The fourth form is the first one for a decode batch: the prompt's state is
forked into B sequences (``fork``) and the batch's decode-step graph is
profiled per step.

The third form times the gated-DeltaNet block alone (``gsq_gdn`` at the
model's 16 key / 48 value heads) for prompts of 1, 16, 128 and 512 tokens:
a CUDA graph of 10 calls, replayed, CUDA events.

Builds the full 27B model (random-init packed weights, the default type
mix), runs a prompt prefill, captures the decode-step graph, and records
``tokens`` graph replays with the CUDA profiler (CUPTI activity records:
device start/end of every kernel, no replay or serialisation).  Prints the
wall time per token (first kernel start to last kernel end) and, per kernel,
the device time and launch count per token.  With programmatic dependent
launch kernels overlap, so the per-kernel times add up to more than the wall
time.
"""
from __future__ import annotations

import sys

import torch
from torch.profiler import ProfilerActivity, profile

from .models import Qwen35Config, build_qwen35, random_weights


def _table(prof, per: int, label: str) -> None:
    kern = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    t0 = min(e.time_range.start for e in kern)
    t1 = max(e.time_range.end for e in kern)
    print(f"wall per {label}: {(t1 - t0) / per:.1f} us")
    rows = sorted(prof.key_averages(), key=lambda e: -e.device_time_total)
    print(f"{'us/' + label:>12} {'launches/' + label:>16} {'us each':>9}  kernel")
    for e in rows:
        if e.device_time_total <= 0:
            continue
        print(f"{e.device_time_total / per:12.1f} {e.count / per:16.1f} "
              f"{e.device_time_total / max(e.count, 1):9.2f}  {e.key[:100]}")


def prefill(prompt: int = 512) -> None:
    """Device time per kernel of one eager prompt prefill."""
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = Qwen35Config()
    model = build_qwen35(random_weights(cfg, dev, seed=0), cfg, dev, max_len=prompt + 16)
    ids = torch.randint(0, cfg.vocab_size, (prompt,), device=dev, dtype=torch.int32)
    model.prefill(ids)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        model.prefill(ids)
        torch.cuda.synchronize()
    _table(prof, 1, "prefill")


def gdn(lengths=(1, 16, 128, 512)) -> None:
    """Device time of one gsq_gdn call (prep + scan + norm kernels; one
    kernel for a single token) at the model's head counts."""
    from . import _lib
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = Qwen35Config()
    nk, nv, d = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_value_head_dim
    C = cfg.gdn_conv_dim
    g = torch.Generator(device=dev).manual_seed(3)
    lib = _lib.load()
    cw = torch.randn(C, 4, device=dev, generator=g) * 0.3
    A = -torch.exp(torch.rand(nv, device=dev, generator=g))
    dtb = torch.randn(nv, device=dev, generator=g) * 0.5
    nw = torch.ones(d, device=dev)
    state = torch.zeros(nv, d, d, device=dev)
    conv = torch.zeros(4, C, device=dev)
    pos = torch.zeros(1, dtype=torch.int32, device=dev)
    for T in lengths:
        proj = torch.randn(T, C + nv * d, device=dev, generator=g)
        ab = torch.randn(T, 2 * nv, device=dev, generator=g).half()
        out = torch.empty(T, nv * d, dtype=torch.float16, device=dev)
        need = lib.gsq_gdn_scratch_bytes(T, nk, nv)
        scratch = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)

        def call():
            _lib.check(lib.gsq_gdn(proj.data_ptr(), proj.stride(0), ab.data_ptr(), ab.stride(0), None, 0, None, 0,
                                   T, nk, nv, conv.data_ptr(), pos.data_ptr(), cw.data_ptr(), A.data_ptr(),
                                   dtb.data_ptr(), nw.data_ptr(), 1e-6, state.data_ptr(),
                                   scratch.data_ptr() if need else None, need, out.data_ptr(),
                                   _lib.DTYPE_CODES[torch.float16], _lib.stream_ptr(dev)))

        call()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream(device=dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            with torch.cuda.graph(graph, stream=st):
                for _ in range(10):
                    call()
        torch.cuda.current_stream(dev).wait_stream(st)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        print(f"gsq_gdn T={T}: {e0.elapsed_time(e1) * 1e3 / 50:.1f} us per call")
    if lib.gsq_device_status(None) != 0:
        raise RuntimeError("device status after the gsq_gdn timing")


def main(prompt: int = 182, tokens: int = 4, batch: int = 1) -> None:
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = Qwen35Config()
    model = build_qwen35(random_weights(cfg, dev, seed=0), cfg, dev, max_len=prompt + tokens + 16, max_batch=batch)
    ids = torch.randint(0, cfg.vocab_size, (prompt,), device=dev, dtype=torch.int32)
    model.prefill(ids)
    if batch > 1:
        model.fork(batch)
    model.decode_step([int(t) for t in torch.randint(0, cfg.vocab_size, (batch,))] if batch > 1 else None)
    model.capture_decode()
    model.replay_decode(3)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        model.replay_decode(tokens)
        torch.cuda.synchronize()
    _table(prof, tokens, "token" if batch == 1 else f"step of {batch}")


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "prefill":
        prefill(*(int(a) for a in sys.argv[2:3]))
    elif len(sys.argv) > 1 and sys.argv[1] == "gdn":
        gdn()
    elif len(sys.argv) > 1 and sys.argv[1] == "batch":
        rest = [int(v) for v in sys.argv[2:5]]
        main(*rest[1:], batch=rest[0] if rest else 8)
    else:
        main(*(int(a) for a in sys.argv[1:3]))
