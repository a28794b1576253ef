#!/usr/bin/env python
"""Headline benchmark: PPO env-steps/s on 65,536 CartPole envs per GPU.

Workload (weak scaling: every rank owns its own 65,536 envs):
  65,536 GPU CartPole envs (dt 0.02, auto-reset, 500-step truncation), rollout
  of 128 steps (8,388,608 transitions per rank per iteration), actor and critic
  MLPs 4-256-256-{2,1} (tanh; bf16 tensor-core GEMMs, fp32 master weights),
  GAE (gamma 0.99, lambda 0.95), 4 epochs of minibatch 32,768 with clip 0.2 and
  Adam 3e-4; with N > 1 GPUs the gradient of every minibatch is reduced across
  ranks (data parallel).
One step = one full PPO iteration (rollout + GAE + 1,024 minibatch updates).
value = N * 65,536 * 128 * K / (max over ranks of the device time of K steps).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--grpo-steps G]

The JSON line also carries the second half of the headline metric under
"grpo": GRPO train tokens/s/box on the 1.5B-shape policy, 64 prompts x 8 per
model replica; on one GPU the whole model, on N >= 2 GPUs tensor parallel
over rank pairs x data parallel over the N/2 pairs (TP2 x DP4 at N = 8).

For N > 1 run under torch.distributed.run (one process per GPU).
``--impl reference`` runs the reference build's own Python API (installed in
baseline/_ref) on its stock PPO example loop at the same env count.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "PPO env-steps/s (64K envs)"
NUM_ENVS = 65536
ROLLOUT = 128
MINIBATCH = 32768
EPOCHS = 4
HIDDEN = (256, 256)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--num-envs", type=int, default=NUM_ENVS)
    p.add_argument("--rollout", type=int, default=ROLLOUT)
    p.add_argument("--dp", choices=["fused", "nccl"], default="fused",
                   help="gradient reduction for N > 1: fused peer-memory kernel or NCCL all-reduce")
    p.add_argument("--grpo-steps", type=int, default=2,
                   help="timed steps of the GRPO measurement (0: skip); 3 warm-up steps")
    return p.parse_args()


def run_grpo(args, world, rank, local):
    """Secondary measurement: GRPO train tokens/s on the 1.5B-shape policy
    (64 prompts x 8 samples per model replica, 256 + 512 tokens), device-timed,
    max over ranks.  One GPU: the whole model on the GPU.  N >= 2 GPUs: the
    layout of the TP2 x DP4 workload, tensor parallel over rank pairs (rollout
    and training on the fused all-gather->GEMM / GEMM->reduce-scatter kernels)
    x data parallel over the N/2 pairs (fused peer-memory optimizer step)."""
    import torch

    from turbol_b200.rl.grpo import GRPOConfig, GRPOTrainer

    cfg = GRPOConfig(num_prompts=64, group_size=8, prompt_len=256, response_len=512, micro_batch=8)
    tp = 2 if world >= 2 else 1
    if world % tp:
        raise ValueError(f"GRPO layout TP{tp} needs an even GPU count, got {world}")
    if tp > 1:
        tr = GRPOTrainer(cfg, f"cuda:{local}", dp="fused", tp=tp, tp_mode="train")
    else:
        tr = GRPOTrainer(cfg, f"cuda:{local}", dp="none")
    replicas = world // tp
    warm = 3
    for _ in range(warm):
        tr.step()
    times = []
    last = None
    for _ in range(args.grpo_steps):
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        last = tr.step()
        e1.record()
        torch.cuda.synchronize()
        times.append(max_over_ranks(e0.elapsed_time(e1) / 1e3, world))
    sec = sum(times) / len(times)
    if hasattr(tr.opt, "check"):
        tr.opt.check()
    if tp > 1:
        tr.comm.check()
    if tr.sync is not None:
        tr.sync.check()
    par = "dp1" if tp == 1 else (f"tp{tp}xdp{replicas}: tensor-parallel training on the fused TP collectives, "
                                 f"fused DP optimizer step over the {replicas} replicas, rollout on a full bf16 "
                                 f"replica per GPU refreshed by the fused weight all-gather")
    out = {"metric": "GRPO train tokens/s/box", "value": replicas * cfg.batch * cfg.seq_len / sec,
           "unit": "tokens/s", "n_gpus": world, "steps": args.grpo_steps, "warmup": warm, "s_per_step": sec,
           "phases_s": {k: last[k] for k in ("rollout_s", "reward_ref_s", "train_s")},
           "config": {"model": "qwen2-1.5b-shape decoder (28 layers, hidden 1536, 12q/2kv heads, ffn 8960, "
                               "vocab 151936)", "prompts_per_replica": cfg.num_prompts, "group": cfg.group_size,
                      "prompt_len": cfg.prompt_len, "response_len": cfg.response_len,
                      "global_batch_sequences": replicas * cfg.batch, "parallelism": par},
           "scaling": "weak", "timing": "CUDA events around each step, max over ranks"}
    del tr
    torch.cuda.empty_cache()
    return out


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons every 200 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.t is not None:
            self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def run_ours(args):
    import torch

    sys.path.insert(0, ROOT)
    from turbol_b200.rl.ppo import PPOConfig, PPOTrainer

    rank, world, local = dist_setup(args.gpus)
    cfg = PPOConfig(num_envs=args.num_envs, rollout_steps=args.rollout, hidden=HIDDEN, epochs=EPOCHS,
                    minibatch_size=MINIBATCH, lr=3e-4, clip=0.2, seed=1, compute_dtype="bf16", cuda_graphs=True)
    tr = PPOTrainer(cfg, device=f"cuda:{local}", rank=rank, dp=args.dp if world > 1 else "none")
    for _ in range(args.warmup):
        tr.train_iteration()
    tr.metrics()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    start.record()
    for _ in range(args.steps):
        tr.train_iteration()
    end.record()
    barrier(world)
    ms_dev = start.elapsed_time(end)
    m = tr.metrics()
    # ---- end to end through the public API: per step, H2D of the step's input
    # (the iteration index that keys every RNG stream, from pinned memory) and a
    # D2H read of the step's metrics.
    pinned = torch.empty(1, dtype=torch.int64, pin_memory=True)
    barrier(world)
    t0 = time.perf_counter()
    for k in range(args.steps):
        pinned[0] = tr.iteration
        tr.iter_t.copy_(pinned, non_blocking=True)
        tr.train_iteration()
        em = tr.metrics()  # D2H read of the step result (synchronizes)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    clk = clocks.stop()
    ms_dev = max_over_ranks(ms_dev, world)
    e2e_s = max_over_ranks(e2e_s, world)
    steps_total = world * cfg.batch * args.steps
    value = steps_total / (ms_dev / 1e3)
    e2e_value = steps_total / e2e_s
    tr.check_collectives()
    # our kernels per iteration: rollout step = MLP forward (first layer + 2 GEMMs)
    # + fused act/env-step kernel; observation pad + bootstrap forward (3); GAE 1;
    # per minibatch: gather, first layer, 2 forward GEMMs, loss,
    # dW3 and dZ2 passes (2 kernels each), 4 backward GEMMs + 3 split-K reduces,
    # optimizer (Adam or the fused DP kernel), counter; end counter
    per_mb = 1 + 1 + 2 + 1 + 4 + 4 + 3 + 1 + 1
    launches_per_iter = cfg.rollout_steps * 4 + 1 + 3 + 1 + cfg.epochs * cfg.n_minibatches * per_mb + 1
    out = {
        "metric": METRIC, "value": value, "unit": "env-steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_dev / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (on-device CartPole simulation, random-init weights)",
        "config": {"model": "CartPole PPO actor-critic MLP 4-256-256-{2,1} tanh",
                   "global_batch": world * cfg.batch, "seq_len": cfg.rollout_steps,
                   "num_envs_per_gpu": cfg.num_envs, "minibatch": cfg.minibatch_size, "epochs": cfg.epochs,
                   "parallelism": f"dp{world}", "dp_reduction": args.dp if world > 1 else "none",
                   "l2": "inputs larger than L2 (rollout storage ~310 MB per iteration per GPU)"},
        "clocks": clk,
        "e2e": {"value": e2e_value, "unit": "env-steps/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 8 * 4 + 8 * 4},
        "gpu_launches": launches_per_iter * args.steps,
        "final_mean_return": m.get("mean_return"),
    }
    tr.release_graphs()
    del tr
    torch.cuda.empty_cache()
    if args.grpo_steps > 0:
        try:
            out["grpo"] = run_grpo(args, world, rank, local)
        except Exception as e:  # the headline line is printed regardless
            out["grpo"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()


def run_reference(args):
    """The reference's own PPO example loop (turbol_vllm/examples/py/ppo_example.py:146-210) through its
    public API at 65,536 envs: per step, random actions -> env.step -> reward.to_numpy -> push_batch.
    Its only throughput notion is that loop's fps (ppo_example.py:195), so one step is one such env step."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "turbol")):
        print(json.dumps({"impl": "reference", "unavailable": "reference build not installed in baseline/_ref "
                          "(run baseline/build_reference.sh)"}))
        return
    import numpy as np
    import torch

    sys.path.insert(0, ref_dir)
    import turbol  # the reference package

    rank, world, local = dist_setup(args.gpus)
    dev = f"cuda:{local}"
    N, obs_dim, act_dim = args.num_envs, 4, 2
    env = turbol.GPUEnvironment(num_envs=N, obs_dim=obs_dim, act_dim=act_dim, device=dev)
    env.reset()
    buf = turbol.RingBuffer(capacity=args.rollout * N, obs_dim=obs_dim, act_dim=act_dim, device=dev)
    rng = np.random.default_rng(1)

    def random_action():
        arr = np.clip(rng.standard_normal((N, act_dim)).astype(np.float32), -1.0, 1.0)
        t = turbol.Tensor((N, act_dim), "float32", "cpu")
        t.to_numpy()[:] = arr
        t.to_device(dev)
        return t

    obs = env.observe()

    def step():
        nonlocal obs
        a = random_action()
        nobs, r, d = env.step(a)
        np.asarray(r.to_numpy())
        buf.push_batch(obs, a, r, d)
        obs = nobs

    for _ in range(args.warmup):
        step()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    barrier(world)
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    ms = max_over_ranks(start.elapsed_time(end), world)
    wall = max_over_ranks(wall, world)
    value = world * N * args.steps / (ms / 1e3)
    out = {"impl": "reference", "metric": METRIC, "value": value, "unit": "env-steps/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
           "data": "synthetic (reference linear env, random actions)",
           "config": {"model": "reference ppo_example loop (LinearEnv obs 4 act 2, RingBuffer push_batch)",
                      "global_batch": world * N, "seq_len": args.rollout, "parallelism": f"dp{world}",
                      "note": "the reference has no CartPole and no PPO update; its example's fps counts env.step + "
                              "push_batch only", "l2": "inputs larger than L2 (ring buffer 25 MB+ per step written)"},
           "clocks": clk, "e2e": {"value": world * N * args.steps / wall, "unit": "env-steps/s",
                                  "h2d_bytes_per_step": N * act_dim * 4, "d2h_bytes_per_step": N * 4},
           "gpu_launches": None}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
