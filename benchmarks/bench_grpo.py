#!/usr/bin/env python
"""GRPO training throughput on one GPU (Qwen2-1.5B-shaped policy, random init).

Workload: 64 prompts of 256 uniform-random token ids x group 8, responses of
512 tokens sampled at temperature 1.0, hash reward, group-normalized
advantages, clip 0.2, KL 0.04 to a frozen reference copy, one Adam update per
step.  Prints one JSON line: train tokens/s = 512 * 768 tokens / step time,
with the rollout / reward+reference / train phase times.

  python benchmarks/bench_grpo.py [--steps K] [--warmup W] [--prompts P] [--tiny]
  torchrun --nproc-per-node N benchmarks/bench_grpo.py --gpus N [--dp fused|nccl] [--tp T [--tp-mode M]]
      (data parallel: --prompts per GPU; with --tp, per tensor-parallel group; tokens/s is the whole job's)
"""
import argparse
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1, help="data-parallel ranks (launch with torchrun for > 1)")
    ap.add_argument("--dp", choices=["fused", "nccl"], default="fused")
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel group size")
    ap.add_argument("--tp-mode", choices=["train", "rollout"], default="train",
                    help="train: TP rollout and TP training (TP x DP); rollout: TP rollout, data-parallel training")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--prompts", type=int, default=64, help="prompts per rank")
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=256)
    ap.add_argument("--response-len", type=int, default=512)
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--tiny", action="store_true")
    a = ap.parse_args()
    import datetime

    import torch
    import torch.distributed as dist

    from turbol_b200.models.llm import LMConfig
    from turbol_b200.rl.grpo import GRPOConfig, GRPOTrainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}: launch with torchrun --nproc-per-node {a.gpus}")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dp = "none"
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        dp = a.dp
    rank = dist.get_rank() if world > 1 else 0
    cfg = GRPOConfig(model=LMConfig.tiny() if a.tiny else LMConfig.qwen2_1p5b(), num_prompts=a.prompts,
                     group_size=a.group, prompt_len=a.prompt_len, response_len=a.response_len,
                     micro_batch=a.micro_batch)
    if a.tp > 1 and (world < 2 or world % a.tp):
        raise SystemExit("--tp needs a world size that is a multiple of it")
    tr = GRPOTrainer(cfg, str(dev), dp=dp, tp=a.tp, tp_mode=a.tp_mode)
    for _ in range(a.warmup):
        tr.step()
    times, last = [], None
    for _ in range(a.steps):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        last = tr.step()
        t1.record()
        torch.cuda.synchronize(dev)
        ms = torch.tensor([t0.elapsed_time(t1)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        times.append(ms.item() / 1e3)
    sec = sum(times) / len(times)
    if rank == 0:
        groups = world // a.tp  # each tensor-parallel group trains on its own prompts
        out = {"metric": "GRPO train tokens/s", "value": groups * cfg.batch * cfg.seq_len / sec, "unit": "tokens/s",
               "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "s_per_step": sec,
               "higher_is_better": True, "scaling": "weak", "dtype": "bf16",
               "data": "synthetic (random prompt ids, random-init weights)",
               "phases_s": {k: last[k] for k in ("rollout_s", "reward_ref_s", "train_s")},
               "decode_tokens_per_s": groups * cfg.batch * cfg.response_len / last["rollout_s"],
               "config": {"model": "qwen2-1.5b-shape" if not a.tiny else "tiny", "prompts_per_group": cfg.num_prompts,
                          "group": cfg.group_size, "prompt_len": cfg.prompt_len, "response_len": cfg.response_len,
                          "micro_batch": cfg.micro_batch, "params": cfg.model.param_count(),
                          "parallelism": ((f"tp{a.tp}xdp{groups} rollout and training" if a.tp_mode == "train"
                                           else f"tp{a.tp}xdp{groups} rollout, dp{world} training") if a.tp > 1
                                          else f"dp{world}") + (f" ({dp})" if world > 1 else "")},
               "timing": "CUDA events around each step, max over ranks",
               "reward_mean": last["reward_mean"], "kl": last["kl"],
               "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 2**30}
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
