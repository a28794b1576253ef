"""Worker for the multi-GPU data-parallel tests (launched by test_dp_multigpu.py
under torch.distributed.run, one process per GPU).  Checks:
  1. the peer-memory all-reduce against the arithmetic result;
  2. the fused all-reduce + Adam kernels (ZeRO-1 and replicated one-handshake)
     against all-reduce + the fp32 Adam oracle;
  3. PPO with the fused data-parallel step keeps identical weights on all ranks
     and matches the NCCL path after one iteration.
Exits non-zero on any mismatch."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200.ops import reference as ref  # noqa: E402
from turbol_b200.parallel.peer import FusedDataParallelAdam, PeerBuffers  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)

    # 1. all-reduce
    n = 100003
    pb = PeerBuffers(n * 4, None)
    buf = pb.tensor(0, n, torch.float32)
    for it in range(3):
        buf.copy_(torch.arange(n, device=dev, dtype=torch.float32) * (rank + 1) + it)
        pb.mem.allreduce(0, 0, n, 1.0)
        torch.cuda.synchronize()
        exp = torch.arange(n, device=dev, dtype=torch.float32) * sum(range(1, world + 1)) + it * world
        assert torch.allclose(buf, exp, rtol=1e-6), f"allreduce mismatch on rank {rank}"
    pb.check()

    # 2. fused all-reduce + Adam vs all-reduce + oracle Adam, in both modes
    #    (ZeRO-1 reduce-scatter / all-gather, and the replicated one-handshake step)
    m = 65541
    for replicated in (False, True):
        opt = FusedDataParallelAdam(m, None, lr=1e-3, replicated=replicated)
        g0 = torch.Generator().manual_seed(0)
        init = torch.randn(m, generator=g0)
        opt.param.copy_(init.to(dev))
        opt.shadow.copy_(opt.param)
        p_ref = init.clone().double()
        m_ref, v_ref = torch.zeros(m, dtype=torch.float64), torch.zeros(m, dtype=torch.float64)
        for step in range(1, 5):
            grads = [torch.randn(m, generator=torch.Generator().manual_seed(100 * step + r)) for r in range(world)]
            opt.grad.copy_(grads[rank].to(dev))
            opt.step()
            torch.cuda.synchronize()
            gmean = sum(g.double() for g in grads) / world
            ref.adam_step(p_ref, gmean, m_ref, v_ref, step, 1e-3)
            assert torch.allclose(opt.param.cpu().double(), p_ref, atol=2e-6), \
                f"fused adam mismatch rank {rank} (replicated={replicated}, step {step})"
            assert torch.allclose(opt.shadow.float().cpu(), opt.param.cpu(), atol=1e-2, rtol=1e-2)
        opt.check()
        # replicated: every rank computed the same weights, bit for bit
        ws = [torch.empty_like(opt.param) for _ in range(world)]
        dist.all_gather(ws, opt.param)
        for other in ws:
            assert torch.equal(other, opt.param), f"rank {rank}: weights differ across ranks (replicated={replicated})"

    # 3. PPO: weights identical across ranks after fused-DP iterations
    from turbol_b200.rl.ppo import PPOConfig, PPOTrainer

    cfg = PPOConfig(num_envs=2048, rollout_steps=16, hidden=(64, 64), epochs=2, minibatch_size=8192, seed=1)
    tr = PPOTrainer(cfg, device=str(dev), rank=rank, dp="fused")
    for _ in range(3):
        tr.train_iteration()
    torch.cuda.synchronize()
    tr.check_collectives()
    w = tr.net.flat.clone()
    ws = [torch.empty_like(w) for _ in range(world)]
    dist.all_gather(ws, w)
    for other in ws:
        assert torch.equal(other, w), f"rank {rank}: weights diverged across ranks"
    tr.release_graphs()
    dist.barrier()
    if rank == 0:
        print("DP_WORKER_OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
