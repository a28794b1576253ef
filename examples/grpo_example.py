"""GRPO on a decoder-only policy with the turbol_b200 rollout engine and trainer.

Same command line as the reference example (turbol_vllm/examples/py/grpo_example.py:45-60):
    python examples/grpo_example.py --num-prompts 32 --max-tokens 128 --num-steps 100

The reference echoes prompts through its rollout engine and updates a linear
policy on a dummy batch (grpo_example.py:124-151); this runs GRPO: the policy
samples G responses per prompt with its own paged-KV decode loop, rewards are
scored (the hash reward by default, or the RewardEngine's rule reward on the
decoded bytes), advantages are normalized within each group, and the policy
takes a clipped-ratio step with a k3 KL penalty against a frozen reference.

``--model`` picks a random-init architecture ("tiny" runs anywhere with a GPU
in seconds; "qwen2-1.5b" is the 28-layer, 1536-hidden shape); ``--model-path``
is accepted for command-line compatibility and only names the run.

On several GPUs (one process per GPU):
    torchrun --nproc-per-node 8 examples/grpo_example.py --model qwen2-1.5b --tp 2 --dp fused
runs tensor-parallel groups of --tp ranks (rollout and training) with data
parallelism across the groups.
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile
import time

import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))

import turbol_b200 as turbol  # noqa: E402


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="turbol_b200 GRPO example")
    p.add_argument("--model-path", type=str, default="", help="accepted for compatibility; weights are random-init")
    p.add_argument("--num-prompts", type=int, default=32)
    p.add_argument("--max-tokens", type=int, default=128, help="response length")
    p.add_argument("--temperature", type=float, default=1.0)
    p.add_argument("--num-steps", type=int, default=100)
    p.add_argument("--lr", type=float, default=1e-4)
    p.add_argument("--kl-coef", type=float, default=0.01)
    p.add_argument("--device", type=str, default="cuda:0")
    p.add_argument("--log-dir", type=str, default="")
    p.add_argument("--print-every", type=int, default=10)
    # additions
    p.add_argument("--model", choices=["tiny", "qwen2-1.5b", "llama3-8b"], default="tiny")
    p.add_argument("--group-size", type=int, default=8)
    p.add_argument("--prompt-len", type=int, default=64)
    p.add_argument("--micro-batch", type=int, default=8)
    p.add_argument("--clip", type=float, default=0.2)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--dp", choices=["fused", "nccl"], default="fused",
                   help="data-parallel gradient reduction when launched on several GPUs (torchrun)")
    p.add_argument("--tp", type=int, default=1, help="tensor-parallel group size (rollout and training)")
    p.add_argument("--checkpoint-dir", type=str, default="")
    p.add_argument("--checkpoint-every", type=int, default=0)
    return p.parse_args(argv)


def main(argv=None):
    args = parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("GRPO runs the sm_100a kernels: a CUDA device is required")
    from turbol_b200.models.llm import LMConfig
    from turbol_b200.rl.grpo import GRPOConfig, GRPOTrainer

    model = {"tiny": LMConfig.tiny(n_layers=4), "qwen2-1.5b": LMConfig.qwen2_1p5b(),
             "llama3-8b": LMConfig.llama3_8b()}[args.model]
    cfg = GRPOConfig(model=model, num_prompts=args.num_prompts, group_size=args.group_size,
                     prompt_len=args.prompt_len, response_len=args.max_tokens, temperature=args.temperature,
                     lr=args.lr, clip=args.clip, kl_coef=args.kl_coef, micro_batch=args.micro_batch, seed=args.seed)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = 0
    if world > 1:  # launched by torchrun: one process per GPU, TP groups of --tp ranks, DP over the rest
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        args.device = f"cuda:{local}"
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device(args.device))
        rank = dist.get_rank()
        tr = GRPOTrainer(cfg, args.device, dp=args.dp, tp=args.tp)
    else:
        if args.tp > 1:
            raise SystemExit("--tp needs several GPUs: launch with torchrun --nproc-per-node N")
        tr = GRPOTrainer(cfg, args.device)
    if rank != 0:
        args.print_every = 1 << 30
    log_dir = args.log_dir or tempfile.mkdtemp(prefix="turbol_grpo_")
    os.makedirs(log_dir, exist_ok=True)
    tb = turbol.TensorBoardWriter(log_dir)
    print(f"GRPO: model {args.model} ({model.param_count() / 1e6:.1f}M params), {cfg.num_prompts} prompts x G "
          f"{cfg.group_size}, prompt {cfg.prompt_len} + response {cfg.response_len} tokens, device {args.device}")
    for step in range(args.num_steps):
        t0 = time.perf_counter()
        st = tr.step()
        dt = time.perf_counter() - t0
        tok_s = cfg.batch * cfg.seq_len / dt
        scalars = {"grpo/mean_reward": st["reward_mean"], "grpo/reward_std": st["reward_std"],
                   "grpo/pg_loss": st["pg_loss"], "grpo/kl": st["kl"], "grpo/kl_coef": cfg.kl_coef,
                   "grpo/gen_ms": st["rollout_s"] * 1e3, "grpo/reward_ms": st["reward_ref_s"] * 1e3,
                   "grpo/policy_ms": st["train_s"] * 1e3, "grpo/train_tokens_per_s": tok_s}
        for k, v in scalars.items():
            tb.add_scalar(k, float(v), step + 1)
        if (step + 1) % args.print_every == 0 or step + 1 == args.num_steps:
            print(f"step {step + 1:4d}  reward {st['reward_mean']:.4f} +- {st['reward_std']:.4f}  "
                  f"kl {st['kl']:.5f}  pg {st['pg_loss']:+.4f}  gen {st['rollout_s'] * 1e3:7.1f} ms  "
                  f"policy {st['train_s'] * 1e3:7.1f} ms  {tok_s:,.0f} tok/s")
        if args.checkpoint_dir and args.checkpoint_every and (step + 1) % args.checkpoint_every == 0:
            turbol.save_checkpoint(args.checkpoint_dir, step + 1, tr, background=True).wait()
    tb.flush()
    if rank == 0:
        print(f"logs: {log_dir}")
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return tr


if __name__ == "__main__":
    main()
