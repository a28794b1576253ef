#!/usr/bin/env python
"""Data-parallel optimizer step: the fused NVLink kernel vs NCCL + fused Adam.

  torchrun --nproc-per-node N benchmarks/bench_dp_step.py [--numel 1543714304] [--reps 10]

Fused: one kernel per step reduces the fp32 gradient by peer loads
(reduce-scatter), runs Adam on the shard this rank owns and writes the fp32
weights and their bf16 copy into every rank (all-gather by peer stores).
Baseline: NCCL all-reduce (sum) of the fp32 gradient, then the local fused Adam
kernel over all weights.  CUDA events, max over ranks.  The roofline is the
slower of (the step's HBM bytes at the measured copy bandwidth) and (the
bytes this rank sends over NVLink at 770 GB/s per direction):
each rank sends, per element, (W-1)/W of its gradient (4 B) to the owners, and
the owner sends its updated fp32 weight (4 B) and bf16 copy (2 B) to W-1 peers.
For vectors up to REPLICATED_MAX_NUMEL the replicated one-handshake step is
timed too (every rank reads the W-1 peers' whole gradients, 4 B each, and
updates the whole vector locally).
"""
import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200.ops.rl import FusedAdam  # noqa: E402
from turbol_b200.parallel.peer import REPLICATED_MAX_NUMEL, FusedDataParallelAdam  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--numel", type=int, default=1_543_714_304, help="parameters (default: the 1.5B GRPO policy)")
    ap.add_argument("--reps", type=int, default=10)
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    n = a.numel

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = torch.tensor([s.elapsed_time(e) / a.reps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item()

    opt = FusedDataParallelAdam(n, None, lr=1e-6, replicated=False)
    opt.grad.normal_()
    fused_ms = timed(opt.step)
    opt.check()
    del opt
    torch.cuda.empty_cache()
    rep_ms = None
    if n <= REPLICATED_MAX_NUMEL:  # the one-handshake step (every rank pulls every gradient, full Adam)
        opt = FusedDataParallelAdam(n, None, lr=1e-6, replicated=True)
        opt.grad.normal_()
        rep_ms = timed(opt.step)
        opt.check()
        del opt
        torch.cuda.empty_cache()
    p = torch.zeros(n, device=dev)
    g = torch.randn(n, device=dev)
    sh = torch.zeros(n, device=dev, dtype=torch.bfloat16)
    base = FusedAdam(p, g, lr=1e-6, shadow=sh)

    def nccl_step():
        dist.all_reduce(g)
        base.step(grad_scale=1.0 / world)
    nccl_ms = timed(nccl_step)
    if rank == 0:
        link = 770e9
        nvlink_bytes = n * 4 * (world - 1) / world + n * (4 + 2) * (world - 1) / world
        # HBM traffic for this rank's shard: its gradient read from every rank (4 B each),
        # m and v read and written (16 B), the fp32 weight read and written (8 B), and the
        # updated fp32 + bf16 weight written into every rank (6 B each)
        hbm_bytes = n / world * (4 * world + 16 + 8 + 6 * world)
        roof_ms = max(nvlink_bytes / link, hbm_bytes / 6.56e12) * 1e3
        print(json.dumps({"benchmark": "dp_optimizer_step", "world": world, "numel": n,
                          "fused_ms": fused_ms, "fused_replicated_ms": rep_ms,
                          "replicated_nvlink_bytes_per_rank": n * 4 * (world - 1),
                          "nccl_allreduce_plus_adam_ms": nccl_ms,
                          "roofline_ms": roof_ms, "fused_frac_of_roofline": roof_ms / fused_ms,
                          "nvlink_bytes_per_rank": nvlink_bytes, "timing": "CUDA events, max over ranks"}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
