#!/usr/bin/env python
"""PPO-RLHF throughput on a pipeline-parallel policy with a value head.

Default workload: Llama-3-8B-shaped policy (32 layers, hidden 4096, 32 query /
8 KV heads, SwiGLU 14,336, vocab 128,256, RoPE 5e5, bf16, random init), a
linear value head on the trunk, 32 prompts of 512 random ids with 1024-token
responses per step, pipeline micro-batches of 4 sequences (8 micro-batches,
1F1B over NCCL send/recv), weights synced from the trainer stages to every
rank's rollout copy before each step.

    torchrun --nproc-per-node N benchmarks/bench_rlhf_pp.py --gpus N [--tp T] [--steps K] [--warmup W] [--tiny]

With --tp T the N ranks form N / T pipeline stages of T tensor-parallel ranks.

Prints one JSON line: train tokens/s = 32 * 1536 / step time (CUDA events,
max over ranks), with the phase times.
"""
import argparse
import datetime
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=2)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--prompts", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--response-len", type=int, default=1024)
    ap.add_argument("--micro-batch", type=int, default=4)
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel ranks per pipeline stage (PP x TP)")
    ap.add_argument("--tiny", action="store_true")
    a = ap.parse_args()
    import torch
    import torch.distributed as dist

    from turbol_b200.models.llm import LMConfig
    from turbol_b200.rl.ppo_rlhf import PPORLHFTrainer, RLHFConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != a.gpus or world < 1:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}: launch with torchrun --nproc-per-node {a.gpus}")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29581")
    os.environ.setdefault("RANK", "0")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    rank = dist.get_rank()
    cfg = RLHFConfig(model=LMConfig.tiny(n_layers=4) if a.tiny else LMConfig.llama3_8b(), num_prompts=a.prompts,
                     prompt_len=a.prompt_len, response_len=a.response_len, micro_batch=a.micro_batch)
    tr = PPORLHFTrainer(cfg, dev, tp=a.tp)
    for _ in range(a.warmup):
        tr.step()
    times, last = [], None
    for _ in range(a.steps):
        dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        last = tr.step()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        times.append(ms.item() / 1e3)
    sec = sum(times) / len(times)
    if rank == 0:
        print(json.dumps({
            "metric": "PPO-RLHF train tokens/s", "value": cfg.num_prompts * cfg.seq_len / sec, "unit": "tokens/s",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "s_per_step": sec, "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic (random prompt ids, random-init weights)",
            "phases_s": {k: last[k] for k in ("sync_s", "rollout_s", "score_s", "train_s")},
            "config": {"model": "llama3-8b-shape" if not a.tiny else "tiny", "prompts": cfg.num_prompts,
                       "prompt_len": cfg.prompt_len, "response_len": cfg.response_len,
                       "micro_batch": cfg.micro_batch, "parallelism": f"pp{world // a.tp} (1F1B, NCCL p2p)" + (
                           f" x tp{a.tp} (fused AG-GEMM / GEMM-RS)" if a.tp > 1 else ""),
                       "params": cfg.model.param_count()},
            "timing": "CUDA events around each step, max over ranks",
            "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 2**30}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
