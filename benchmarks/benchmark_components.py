#!/usr/bin/env python
"""Component micro-benchmarks.

Same components and flags as the reference's benchmark_components
(turbol_vllm/benchmarks/benchmark_components.cpp:62-309):
    python benchmarks/benchmark_components.py --device cuda --num-envs 4096 --steps 500 --batch 256
(defaults obs_dim 16, act_dim 4, replay capacity 2^20), reporting env.Step,
RingBuffer PushBatch / Sample, PolicyEngine Forward / Update and GAE.

``--replay-config`` runs the large replay / advantage workload instead:
capacity 16,777,216 x obs 64 (fp32 ~N(0,1)), act 8, rewards ~U(-1,1),
done ~Bernoulli(0.01); push_batch of 65,536 rows; uniform and prioritized
(sum-tree, priorities ~Exp(1), alpha 0.6, beta 0.4) samples of 65,536; GAE
over [256, 65,536] with gamma 0.99, lambda 0.95.

GPU operations are timed with CUDA events on the launching stream (mean over
``--steps`` calls after 3 warm-ups); CPU operations with the host clock.
A final JSON line collects every result.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import turbol_b200 as turbol  # noqa: E402
from turbol_b200.ops import rl as rlops  # noqa: E402


def timed(fn, steps: int, cuda: bool, warmup: int = 3) -> float:
    """Mean milliseconds per call."""
    for _ in range(warmup):
        fn()
    if cuda:
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    return (time.perf_counter() - t0) * 1e3 / steps


def report(results, name, ms, per_call, unit):
    rate = per_call * 1e3 / ms
    results[name] = {"ms": ms, "rate": rate, "unit": unit}
    print(f"  {name:34s} {ms:10.4f} ms/op   {rate:18,.1f} {unit}")


def bench_default(args, dev, cuda, results):
    N, O, A, steps, B = args.num_envs, args.obs_dim, args.act_dim, args.steps, args.batch
    print(f"\n[1/6] GPUEnvironment::Step (linear env, {N} envs, {O}x{A})")
    env = turbol.GPUEnvironment(N, O, A, dev, "linear")
    act = torch.rand(N, A, device=dev) * 2 - 1
    obs, rew, done = torch.empty(N, O, device=dev), torch.empty(N, device=dev), torch.empty(N, dtype=torch.bool,
                                                                                                 device=dev)
    ms = timed(lambda: env.step_into(act, obs, rew, done), steps, cuda)
    report(results, "env_step", ms, N, "env-steps/s")

    print(f"\n[2/6] RingBuffer::PushBatch ({B}/batch, capacity {args.capacity})")
    buf = turbol.RingBuffer(args.capacity, O, A, dev, seed=1)
    ft = turbol.from_torch
    o, a = ft(torch.randn(B, O, device=dev)), ft(torch.randn(B, A, device=dev))
    r, d = ft(torch.randn(B, device=dev)), ft(torch.zeros(B, dtype=torch.bool, device=dev))
    ms = timed(lambda: buf.push_batch(o, a, r, d), steps, cuda)
    report(results, "replay_push_batch", ms, B, "transitions/s")

    print(f"\n[3/6] RingBuffer::Sample ({B}/batch)")
    so, sa, sr, sd = turbol.Tensor(), turbol.Tensor(), turbol.Tensor(), turbol.Tensor()
    ms = timed(lambda: buf.sample(B, so, sa, sr, sd), steps, cuda)
    report(results, "replay_sample", ms, B, "transitions/s")

    print(f"\n[4/6] PolicyEngine::Forward (batch {B})")
    pe = turbol.PolicyEngine(obs_dim=O, act_dim=A, device=dev)
    pe.initialize()
    x = torch.randn(B, O, device=dev)
    ms = timed(lambda: pe.act(x), steps, cuda)
    report(results, "policy_forward", ms, B, "samples/s")

    print(f"\n[5/6] PolicyEngine::Update (batch {B})")
    batch = torch.randn(B, O + A + 2, device=dev)
    ms = timed(lambda: pe.update(batch), steps, cuda)
    report(results, "policy_update", ms, B, "samples/s")

    gae_bench(results, 256, N, steps, dev, cuda, "[6/6]")


def gae_bench(results, T, N, steps, dev, cuda, tag):
    print(f"\n{tag} GAE (T={T}, envs={N})")
    g = torch.Generator().manual_seed(3)
    rew = (torch.rand(T, N, generator=g) * 2 - 1).to(dev)
    val = torch.randn(T + 1, N, generator=g).to(dev)
    done = (torch.rand(T, N, generator=g) < 0.01).to(torch.uint8).to(dev)
    adv, ret = torch.empty(T, N, device=dev), torch.empty(T, N, device=dev)
    scratch = None
    if cuda:
        n = turbol.turbol_core.ops.gae_scratch_numel(T, N)
        scratch = torch.empty(max(n, 1), device=dev)
    ms = timed(lambda: rlops.gae(rew, val, done, 0.99, 0.95, scratch=scratch, out=(adv, ret)), max(10, steps // 5),
               cuda)
    report(results, "gae", ms, T * N, "env-steps/s")


def bench_replay_config(args, dev, cuda, results):
    cap, O, A, B = 16_777_216, 64, 8, 65_536
    steps = max(5, args.steps // 25)
    print(f"\n[1/4] RingBuffer push_batch of {B} rows (capacity {cap:,}, obs {O} fp32, act {A})")
    buf = turbol.PrioritizedReplayBuffer(cap, O, A, alpha=0.6, beta=0.4, device=dev, seed=5)
    g = torch.Generator().manual_seed(7)
    ft = turbol.from_torch
    o = torch.randn(B, O, generator=g).to(dev)
    a = torch.randn(B, A, generator=g).to(dev)
    r = (torch.rand(B, generator=g) * 2 - 1).to(dev)
    d = (torch.rand(B, generator=g) < 0.01).to(dev)
    to, ta, tr_, td = ft(o), ft(a), ft(r), ft(d)
    ms = timed(lambda: buf.push_batch(to, ta, tr_, td), steps, cuda)
    report(results, "replay_push_batch_65536", ms, B, "transitions/s")
    # fill the ring so that sampling covers the whole capacity
    for _ in range(cap // B):
        buf.push_batch(to, ta, tr_, td)
    if cuda:
        torch.cuda.synchronize()
    print(f"\n[2/4] uniform sample of {B}")
    so, sa, sr, sd = turbol.Tensor(), turbol.Tensor(), turbol.Tensor(), turbol.Tensor()
    ms = timed(lambda: buf.sample(B, so, sa, sr, sd), steps, cuda)
    report(results, "replay_sample_uniform_65536", ms, B, "transitions/s")
    print(f"\n[3/4] prioritized sample of {B} (priorities ~Exp(1), alpha 0.6, beta 0.4)")
    idx = torch.arange(cap, device=dev, dtype=torch.int64)
    pr = torch.empty(cap).exponential_(1.0, generator=g).to(dev)
    buf.update_priorities(idx, pr)
    ms = timed(lambda: buf.sample_prioritized(B, 0.4), steps, cuda)
    report(results, "replay_sample_per_65536", ms, B, "transitions/s")
    gae_bench(results, 256, 65_536, args.steps, dev, cuda, "[4/4]")


def main():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--device", default="cuda", choices=["cpu", "cuda"])
    p.add_argument("--num-envs", type=int, default=4096)
    p.add_argument("--obs-dim", type=int, default=16)
    p.add_argument("--act-dim", type=int, default=4)
    p.add_argument("--steps", type=int, default=500)
    p.add_argument("--batch", type=int, default=256)
    p.add_argument("--capacity", type=int, default=1 << 20)
    p.add_argument("--replay-config", action="store_true", help="the 16.7M-capacity replay / GAE workload")
    args = p.parse_args()
    cuda = args.device == "cuda" and torch.cuda.is_available()
    dev = "cuda:0" if cuda else "cpu"
    print("=== turbol_b200 component micro-benchmarks ===")
    print(f"  device {dev}  num_envs {args.num_envs}  obs/act {args.obs_dim}/{args.act_dim}  steps {args.steps}  "
          f"batch {args.batch}")
    results = {}
    if args.replay_config:
        bench_replay_config(args, dev, cuda, results)
    else:
        bench_default(args, dev, cuda, results)
    print(json.dumps({"benchmark": "components", "device": dev, "replay_config": args.replay_config,
                      "timing": "CUDA events, mean per call after 3 warm-ups" if cuda else "host clock",
                      "results": results}))


if __name__ == "__main__":
    main()
