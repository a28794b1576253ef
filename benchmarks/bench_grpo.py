#!/usr/bin/env python
"""GRPO training throughput on one GPU (Qwen2-1.5B-shaped policy, random init).

Workload: 64 prompts of 256 uniform-random token ids x group 8, responses of
512 tokens sampled at temperature 1.0, hash reward, group-normalized
advantages, clip 0.2, KL 0.04 to a frozen reference copy, one Adam update per
step.  Prints one JSON line: train tokens/s = 512 * 768 tokens / step time,
with the rollout / reward+reference / train phase times.

  python benchmarks/bench_grpo.py [--steps K] [--warmup W] [--prompts P] [--tiny]
"""
import argparse
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--prompts", type=int, default=64)
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=256)
    ap.add_argument("--response-len", type=int, default=512)
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--tiny", action="store_true")
    a = ap.parse_args()
    import torch

    from turbol_b200.models.llm import LMConfig
    from turbol_b200.rl.grpo import GRPOConfig, GRPOTrainer

    cfg = GRPOConfig(model=LMConfig.tiny() if a.tiny else LMConfig.qwen2_1p5b(), num_prompts=a.prompts,
                     group_size=a.group, prompt_len=a.prompt_len, response_len=a.response_len,
                     micro_batch=a.micro_batch)
    tr = GRPOTrainer(cfg, "cuda:0")
    for _ in range(a.warmup):
        tr.step()
    times, last = [], None
    for _ in range(a.steps):
        last = tr.step()
        times.append(last["step_s"])
    sec = sum(times) / len(times)
    out = {"metric": "GRPO train tokens/s", "value": cfg.batch * cfg.seq_len / sec, "unit": "tokens/s", "n_gpus": 1,
           "steps": a.steps, "warmup": a.warmup, "s_per_step": sec,
           "phases_s": {k: last[k] for k in ("rollout_s", "reward_ref_s", "train_s")},
           "decode_tokens_per_s": cfg.batch * cfg.response_len / last["rollout_s"],
           "config": {"model": "qwen2-1.5b-shape" if not a.tiny else "tiny", "prompts": cfg.num_prompts,
                      "group": cfg.group_size, "prompt_len": cfg.prompt_len, "response_len": cfg.response_len,
                      "micro_batch": cfg.micro_batch, "params": cfg.model.param_count()},
           "reward_mean": last["reward_mean"], "kl": last["kl"],
           "peak_mem_gb": torch.cuda.max_memory_allocated() / 2**30}
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
