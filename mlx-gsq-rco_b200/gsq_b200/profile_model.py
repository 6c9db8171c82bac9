"""Per-kernel device time of one decode token of the Qwen3.5-hybrid harness.

    python -m gsq_b200.profile_model [prompt_tokens] [tokens]
    python -m gsq_b200.profile_model prefill [prompt_tokens]

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
    _table(prof, tokens, "token")


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "prefill":
        prefill(*(int(a) for a in sys.argv[2:3]))
    else:
        main(*(int(a) for a in sys.argv[1:3]))
