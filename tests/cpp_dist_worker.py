"""Worker for the C++ distributed runtime test (torchrun, 2 GPUs).

Drives turbol_core.dist (turbol/distributed.hpp) without torch.distributed:
the NcclCommunicator bootstraps over the native TCP store, then all-reduce
(sum, mean; fp32 and bf16), all-gather, reduce-scatter, broadcast, a grouped
send/recv exchange and barrier; the DistributedTrainer facade; and the 1F1B
PipelineTrainer over two stages of a two-matrix linear model, with and without
activation recomputation, against the gradients of the same model computed
whole on one GPU."""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import turbol_b200  # noqa: E402

C = turbol_b200.turbol_core
D = C.dist


def ok(st, what):
    assert st.ok(), (what, repr(st))


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    port = int(os.environ["TB_CPP_PORT"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = D.NcclCommunicator()
    ok(comm.initialize(rank, world, local, "127.0.0.1", port, 60.0), "init")
    assert comm.rank == rank and comm.world_size == world
    total = sum(range(1, world + 1))
    t = torch.full((1000,), float(rank + 1), device=dev)
    ok(comm.all_reduce(t, "sum"), "all_reduce sum")
    assert torch.all(t == total)
    t = torch.full((999,), float(rank + 1), device=dev, dtype=torch.bfloat16)
    ok(comm.all_reduce(t, "mean"), "all_reduce mean")
    assert torch.allclose(t.float(), torch.full_like(t.float(), total / world))
    g_in = torch.arange(6, device=dev, dtype=torch.float32) + 10 * rank
    g_out = torch.empty(6 * world, device=dev)
    ok(comm.all_gather(g_in, g_out), "all_gather")
    assert torch.equal(g_out, torch.cat([torch.arange(6, device=dev).float() + 10 * r for r in range(world)]))
    rs_in = torch.arange(4 * world, device=dev, dtype=torch.float32) * (rank + 1)
    rs_out = torch.empty(4, device=dev)
    ok(comm.reduce_scatter(rs_in, rs_out, "sum"), "reduce_scatter")
    assert torch.equal(rs_out, torch.arange(4 * rank, 4 * rank + 4, device=dev).float() * total)
    b = torch.full((17,), float(rank), device=dev)
    ok(comm.broadcast(b, 1), "broadcast")
    assert torch.all(b == 1.0)
    # ring exchange in one group: send to the next rank, receive from the previous one
    s = torch.full((33,), float(rank), device=dev)
    r_ = torch.empty(33, device=dev)
    ok(comm.group_start(), "group_start")
    ok(comm.send(s, (rank + 1) % world), "send")
    ok(comm.recv(r_, (rank - 1) % world), "recv")
    ok(comm.group_end(), "group_end")
    torch.cuda.synchronize()
    assert torch.all(r_ == float((rank - 1) % world))
    ok(comm.barrier(), "barrier")
    # ---- DistributedTrainer facade (its own communicator on another port)
    cfg = D.DistributedConfig()
    cfg.rank, cfg.world_size, cfg.master_port, cfg.device_id = rank, world, port + 1, local
    tr = D.DistributedTrainer(cfg)
    ok(tr.initialize(), "trainer init")
    x = torch.full((5,), float(rank + 1), device=dev)
    ok(tr.all_reduce(x, "mean"), "trainer all_reduce")
    assert torch.allclose(x, torch.full_like(x, total / world))
    y = torch.full((5,), float(rank + 7), device=dev)
    ok(tr.broadcast(y, 0), "trainer broadcast")
    assert torch.all(y == 7.0)
    assert not tr.all_reduce(x, "median").ok()
    ok(tr.barrier(), "trainer barrier")
    ok(tr.shutdown(), "trainer shutdown")
    # ---- PipelineTrainer: stage s computes y = x W_s; loss = 0.5 * mean over the micro-batch of |y|^2
    H, rows, M = 64, 32, 5
    gen = torch.Generator().manual_seed(11)
    W = [(torch.randn(H, H, generator=gen) / H ** 0.5).to(dev) for _ in range(world)]
    X = [torch.randn(rows, H, generator=gen).to(dev) for _ in range(M)]
    # whole-model reference on this GPU
    Wr = [w.clone().requires_grad_() for w in W]
    ref_loss = 0.0
    for i in range(M):
        h = X[i]
        for w in Wr:
            h = h @ w
        loss = 0.5 * (h * h).sum() / rows
        ref_loss += float(loss) / M
        loss.backward()
    for recompute in (False, True):
        grad = torch.zeros(H, H, device=dev)
        keep = {}

        def forward(i, x, _r=recompute):
            if not _r:
                keep[i] = x.clone()
            return x @ W[rank]

        def recomp(i, x):
            keep[i] = x.clone()

        def loss_fn(i, y):
            return float(0.5 * (y * y).sum() / rows), (y / rows).contiguous()

        def backward(i, dy):
            x = keep.pop(i)
            grad.add_(x.t() @ dy)
            return (dy @ W[rank].t()).contiguous()

        pcfg = D.PipelineConfig()
        pcfg.num_pipeline_stages, pcfg.stage_id, pcfg.num_microbatches = world, rank, M
        pcfg.microbatch_batch_sz, pcfg.microbatch_seq_len, pcfg.hidden_size = 1, rows, H
        pcfg.activation_checkpointing = recompute
        pt = D.PipelineTrainer(pcfg)
        ok(pt.initialize(comm, input=(lambda i: X[i]) if rank == 0 else None, forward=forward,
                         loss=loss_fn if rank == world - 1 else None, backward=backward,
                         recompute=recomp if recompute else None, dtype="float32"), "pipeline init")
        st, avg = pt.training_step()
        ok(st, "training_step")
        torch.cuda.synchronize()
        assert torch.allclose(grad, Wr[rank].grad, atol=1e-4, rtol=1e-4), (recompute, (grad - Wr[rank].grad).abs().max())
        if rank == world - 1:
            assert abs(avg - ref_loss) < 1e-3 * max(1.0, abs(ref_loss)), (avg, ref_loss)
        want = [f"{k}{i}" for k, i in C.PipelineSchedule.one_f_one_b(world, rank, M)]
        assert pt.last_order() == want, (pt.last_order(), want)
    ok(comm.barrier(), "final barrier")
    ok(comm.shutdown(), "shutdown")
    if rank == 0:
        print("CPP_DIST_WORKER_OK")


if __name__ == "__main__":
    main()
