#!/usr/bin/env python
"""Trainer -> rollout weight sync of a tensor-parallel trainer: the fused
all-gather into full-model replicas (TPReplicaSync, one kernel of NVLink peer
stores) against NCCL all-gather of the shard buffers + un-sharding copies.

  torchrun --nproc-per-node 2 benchmarks/bench_weight_sync.py [--model qwen2-1.5b|llama3-8b] [--reps 10]

The ranks form groups of --tp (default: all ranks).  CUDA events, mean of
--reps syncs after 2 warm-up syncs, max over ranks.  Roofline: the bytes each
rank sends over NVLink ((tp - 1) x its shard segments) at 770 GB/s per
direction (the measured peer-copy bandwidth of this pool's B200s).
"""
import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200.models.llm import DecoderLM, LMConfig  # noqa: E402
from turbol_b200.models.tp_llm import TPTrainLM  # noqa: E402
from turbol_b200.parallel.dist import build_mesh  # noqa: E402
from turbol_b200.parallel.tp import TensorParallelComm  # noqa: E402
from turbol_b200.parallel.weight_sync import TPReplicaSync  # noqa: E402

LINK_GBS = 770.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2-1.5b", choices=["qwen2-1.5b", "llama3-8b"])
    ap.add_argument("--tp", type=int, default=0)
    ap.add_argument("--reps", type=int, default=10)
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    tp = a.tp or world
    dev = torch.device("cuda", local)
    cfg = LMConfig.qwen2_1p5b() if a.model == "qwen2-1.5b" else LMConfig.llama3_8b()
    mesh = build_mesh(world, rank, tp=tp)
    comm = TensorParallelComm(1024, cfg.hidden, cfg.hidden, group=mesh.tp_group, device=local)
    full = DecoderLM(cfg, dev, seed=0, master=False)
    model = TPTrainLM(full, comm)
    del full
    sync = TPReplicaSync(model, mesh.tp_group)

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(a.reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / a.reps], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    fused_ms = timed(sync)
    sync.check()
    # baseline: NCCL all-gather of every rank's bf16 shard buffer, then the un-sharding copies
    gathered = torch.empty(tp, model.numel, device=dev, dtype=torch.bfloat16)
    target = sync.full

    def nccl_sync():
        dist.all_gather_into_tensor(gathered, model.shadow, group=mesh.tp_group)
        for t in range(tp):
            TPTrainLM.unshard_into(target, gathered[t], model.offsets, tp, t, shards_only=t > 0)

    nccl_ms = timed(nccl_sync)
    roof_ms = sync.bytes_sent / (LINK_GBS * 1e9) * 1e3
    if rank == 0:
        print(json.dumps({"benchmark": "trainer_to_rollout_weight_sync", "model": a.model, "tp": tp,
                          "fused_ms": fused_ms, "nccl_allgather_plus_unshard_ms": nccl_ms,
                          "nvlink_bytes_per_rank": sync.bytes_sent, "roofline_ms": roof_ms,
                          "fused_frac_of_roofline": roof_ms / fused_ms,
                          "timing": "CUDA events, mean of reps, max over ranks"}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
