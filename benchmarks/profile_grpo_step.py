#!/usr/bin/env python
"""Per-kernel device time of one GRPO step, by phase (rollout, reference
log-probs, training), on one GPU.

  python benchmarks/profile_grpo_step.py [--prompts 64] [--tiny]

Builds the bench_grpo trainer (Qwen2-1.5B shape, 64 prompts x 8, 256 + 512
tokens), runs one step to warm up, then runs each phase of one more step under
torch.profiler (CUPTI kernel timestamps) and prints, per phase, the total
kernel time and the kernels that take the most of it (name, calls, time).
Numbers taken under the profiler are for the breakdown only; bench_grpo.py
and bench.py measure the throughput.
"""
import argparse
import collections
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200._native import ops  # noqa: E402
from turbol_b200.models.llm import LMConfig  # noqa: E402
from turbol_b200.rl.grpo import GRPOConfig, GRPOTrainer  # noqa: E402


def table(prof, top: int):
    agg = collections.defaultdict(lambda: [0, 0.0])
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            a = agg[e.name[:90]]
            a[0] += 1
            a[1] += e.device_time_total
    total = sum(v[1] for v in agg.values())
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])[:top]
    return total, rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--prompts", type=int, default=64)
    ap.add_argument("--top", type=int, default=14)
    ap.add_argument("--tiny", action="store_true")
    a = ap.parse_args()
    cfg = GRPOConfig(model=LMConfig.tiny() if a.tiny else LMConfig.qwen2_1p5b(), num_prompts=a.prompts)
    tr = GRPOTrainer(cfg, "cuda:0")
    tr.step()
    torch.cuda.synchronize()
    o = ops()
    from torch.profiler import ProfilerActivity, profile

    phases = {}
    with profile(activities=[ProfilerActivity.CUDA]) as p:
        seqs, _ = tr.gen.generate(tr._prompts(), cfg.group_size, cfg.response_len, cfg.temperature)
        torch.cuda.synchronize()
    phases["rollout"] = p
    resp = seqs[:, cfg.prompt_len:].contiguous()
    lens = torch.full((cfg.batch,), cfg.response_len, device=seqs.device, dtype=torch.int32)
    adv = o.grpo_advantage(o.hash_reward(resp, lens), cfg.group_size, 1e-4, True)
    with profile(activities=[ProfilerActivity.CUDA]) as p:
        ref_lp = tr.ref_logprobs(seqs)
        torch.cuda.synchronize()
    phases["reference log-probs"] = p
    with profile(activities=[ProfilerActivity.CUDA]) as p:
        tr.model.zero_grad()
        tr._train(seqs, ref_lp, adv)
        tr.opt.step()
        torch.cuda.synchronize()
    phases["train (forward, backward, Adam)"] = p
    for name, prof in phases.items():
        total, rows = table(prof, a.top)
        print(f"== {name}: {total / 1e3:.1f} ms of kernel time")
        for k, (n, us) in rows:
            print(f"{us / 1e3:9.2f} ms  {100 * us / total:5.1f}%  x{n:<6d} {k}")


if __name__ == "__main__":
    main()
