#!/usr/bin/env python
"""Per-kernel device times of one PPO minibatch step (CUDA-graph replays).

  python benchmarks/profile_ppo_step.py [--replays 20]

Builds the bench.py PPO trainer (65,536 envs, MLP 4-256-256-{2,1}, minibatch
32,768), runs two iterations, then replays the captured minibatch graph under
torch.profiler (CUPTI kernel timestamps) and prints the time per kernel per
minibatch and the kernels of one replay in order.  Numbers taken under the
profiler are for the breakdown only; bench.py measures the headline.
"""
import argparse
import collections
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200.rl.ppo import PPOConfig, PPOTrainer  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--replays", type=int, default=20)
    a = ap.parse_args()
    cfg = PPOConfig(num_envs=65536, rollout_steps=128, hidden=(256, 256), epochs=4, minibatch_size=32768,
                    cuda_graphs=True)
    tr = PPOTrainer(cfg, device="cuda:0")
    tr.train_iteration()
    tr.train_iteration()
    torch.cuda.synchronize()
    _, mb, _ = tr._graphs
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(a.replays):
            mb[0].replay()
        torch.cuda.synchronize()
    ev = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    agg = collections.defaultdict(list)
    order = []
    for e in ev:
        k = e.name[:70]
        agg[k].append(e.device_time_total)
        if k not in order:
            order.append(k)
    n = a.replays
    print(f"kernel time per minibatch: {sum(sum(v) for v in agg.values()) / n:.1f} us")
    for k in order:
        v = agg[k]
        print(f"{sum(v) / n:8.1f} us/minibatch  x{len(v) / n:4.1f}  {k}")
    per = len(ev) // n
    print("--- one replay")
    for e in ev[:per]:
        print(f"{e.device_time_total:7.1f} us  {e.name[:80]}")


if __name__ == "__main__":
    main()
