"""Worker for the data-parallel GRPO test (2 GPUs, torchrun): after two steps
the fused peer-memory data-parallel path and the NCCL path hold identical
weights on every rank, and agree with each other."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200.models.llm import LMConfig  # noqa: E402
from turbol_b200.rl.grpo import GRPOConfig, GRPOTrainer  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = GRPOConfig(model=LMConfig.tiny(), num_prompts=2, group_size=4, prompt_len=32, response_len=32,
                     micro_batch=4, lr=1e-4)
    finals = {}
    for dp in ("fused", "nccl"):
        tr = GRPOTrainer(cfg, f"cuda:{local}", dp=dp)
        for _ in range(2):
            st = tr.step()
            assert st["tokens"] == cfg.batch * cfg.response_len
        w = tr.model.flat.detach().clone()
        ws = [torch.empty_like(w) for _ in range(world)]
        dist.all_gather(ws, w)
        for r in range(world):
            assert torch.equal(ws[r], ws[0]), (dp, "weights differ across ranks")
        assert torch.equal(tr.model.shadow, tr.model.flat.to(torch.bfloat16)), dp
        finals[dp] = w
        if dp == "fused":
            tr.opt.check()
        del tr
    err = (finals["fused"] - finals["nccl"]).abs().max().item()
    assert err < 1e-5, err
    # tensor-parallel rollout (tp = world) + data-parallel training
    # (row shards of the fused kernels are multiples of 128: 256 sequences per group)
    tcfg = GRPOConfig(model=LMConfig.tiny(), num_prompts=32, group_size=8, prompt_len=32, response_len=16,
                      micro_batch=16, lr=1e-4)
    tr = GRPOTrainer(tcfg, f"cuda:{local}", dp="fused", tp=world, tp_mode="rollout")
    for _ in range(2):
        st = tr.step()
        assert st["tokens"] == tcfg.batch // world * tcfg.response_len
    w = tr.model.flat.detach().clone()
    ws = [torch.empty_like(w) for _ in range(world)]
    dist.all_gather(ws, w)
    assert all(torch.equal(x, ws[0]) for x in ws), "tp: weights differ across ranks"
    # the rollout shard was re-sliced from the updated weights
    assert torch.equal(tr.tpm.w["l0.wo"], tr.model.s["l0.wo"][:, rank * tr.tpm.q_dim:(rank + 1) * tr.tpm.q_dim])
    tr.comm.check()
    del tr
    if rank == 0:
        print("GRPO_DP_WORKER_OK", err)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
