"""Per-kernel device time of one decode token of the Qwen3.5-hybrid harness.

    python -m gsq_b200.profile_model [prompt_tokens] [tokens]

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


def main(prompt: int = 182, tokens: int = 4) -> None:
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = Qwen35Config()
    model = build_qwen35(random_weights(cfg, dev, seed=0), cfg, dev, max_len=prompt + tokens + 16)
    ids = torch.randint(0, cfg.vocab_size, (prompt,), device=dev, dtype=torch.int32)
    model.prefill(ids)
    model.decode_step()
    model.capture_decode()
    model.replay_decode(3)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        model.replay_decode(tokens)
        torch.cuda.synchronize()
    kern = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    t0 = min(e.time_range.start for e in kern)
    t1 = max(e.time_range.end for e in kern)
    print(f"wall per token: {(t1 - t0) / tokens:.1f} us over {tokens} graph replays")
    rows = sorted(prof.key_averages(), key=lambda e: -e.device_time_total)
    print(f"{'us/token':>10} {'launches/token':>15} {'us each':>9}  kernel")
    for e in rows:
        if e.device_time_total <= 0:
            continue
        print(f"{e.device_time_total / tokens:10.1f} {e.count / tokens:15.1f} "
              f"{e.device_time_total / max(e.count, 1):9.2f}  {e.key[:100]}")


if __name__ == "__main__":
    main(*(int(a) for a in sys.argv[1:3]))
