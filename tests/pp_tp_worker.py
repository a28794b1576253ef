"""Worker for pipeline x tensor parallelism (torchrun, 2 or 4 GPUs, TP = 2).

1. A 1F1B pass over TP stages (world / 2 stages of 2 ranks; every rank sends
   its rows to the same TP rank of the next stage) gives the whole model's
   gradients on one GPU: the shards against the slices of the full gradients,
   the replicated tensors after the TP all-reduce.
2. PPO-RLHF with tp=2 runs two steps through the PP x TP trainer; after the
   weight sync every rank's full rollout copy holds the trainer shards."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200._native import ops  # noqa: E402
from turbol_b200.models.llm import DecoderLM, LMConfig  # noqa: E402
from turbol_b200.parallel import pipeline as pp  # noqa: E402
from turbol_b200.parallel.dist import build_mesh  # noqa: E402
from turbol_b200.parallel.tp import TensorParallelComm  # noqa: E402
from turbol_b200.rl.ppo_rlhf import PPORLHFTrainer, RLHFConfig  # noqa: E402

TP = 2


def head_loss_grad(model, x, tgt):
    """d(sum of log p(tgt)) / d x for the rows x (any model with the head)."""
    o = ops()
    N = x.shape[0]
    rstd = torch.empty(N, device=x.device)
    hf = model.final_norm(x, rstd)
    logits = model.logits(hf)
    dlp = torch.full((N,), -1e-3, device=x.device)
    o.logprob(logits, tgt, None, dlp)
    dh = torch.empty_like(hf)
    o.gemm(logits, model.head_weight(), dh, False, True)
    o.gemm(logits, hf, model.head_grad(), True, True, accumulate=True, split_k=1)
    dx = torch.empty_like(x)
    o.rmsnorm_bwd(dh, x, model.f32["norm"], rstd, dx, None, model.g["norm"])
    return dx


def rel(a, b):
    return (a.float() - b.float()).abs().max().item() / (b.float().abs().max().item() + 1e-12)


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = LMConfig.tiny(n_layers=4)
    cfg.tie_embeddings = False
    cfg.init_std = 0.05
    mesh = build_mesh(world, rank, tp=TP, pp=world // TP)
    mb, T, M = 2, 128, 3
    comm = TensorParallelComm(mb * T, cfg.hidden, cfg.hidden, group=mesh.tp_group, device=local)
    # ---- 1. PP x TP gradients == single-GPU gradients
    full = DecoderLM(cfg, dev, seed=5)
    st = pp.PipelineStage(cfg, mesh.pp_rank, mesh.pp, dev, tp_comm=comm)
    st.load_from_full(full)
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, cfg.vocab, (mb * M, T), generator=g).to(dev, torch.int32)
    tgt_all = [torch.roll(ids[i * mb:(i + 1) * mb].reshape(-1), -1).contiguous() for i in range(M)]
    pos = torch.arange(T, device=dev, dtype=torch.int32).repeat(mb)
    full.zero_grad()
    for i in range(M):
        x, saved = full.forward(full.embed(ids[i * mb:(i + 1) * mb]), mb, T, pos, save=True)
        dx = full.backward(head_loss_grad(full, x, tgt_all[i]), saved, mb, T, pos)
        full.embed_backward(ids[i * mb:(i + 1) * mb], dx)
    m = mb * T // TP
    r0 = mesh.tp_rank * m
    pp.set_micro_geometry(mb, T, pos)
    st.zero_grad()
    pp.run_1f1b(st, mesh.pp_ranks, M, m,
                lambda i: st.model.embed_rows(ids[i * mb:(i + 1) * mb].reshape(-1)),
                lambda i, x: head_loss_grad(st.model, x, tgt_all[i][r0:r0 + m].contiguous()),
                lambda i, dx: st.model.embed_backward_rows(ids[i * mb:(i + 1) * mb].reshape(-1), dx),
                group=mesh.pp_group)
    st.model.reduce_replicated_grads()
    torch.cuda.synchronize()
    comm.check()
    tpm = st.model
    Q, KV = cfg.q_dim, cfg.kv_dim
    q0, k0, f0 = tpm.rank * tpm.q_dim, tpm.rank * tpm.kv_dim, tpm.rank * tpm.F
    rows = torch.cat([torch.arange(q0, q0 + tpm.q_dim), torch.arange(Q + k0, Q + k0 + tpm.kv_dim),
                      torch.arange(Q + KV + k0, Q + KV + k0 + tpm.kv_dim)]).to(dev)
    errs = {}
    for name in tpm.offsets:
        kind = name.rsplit(".", 1)[-1]
        ref = full.g[name]
        if kind in ("wqkv", "bqkv"):
            ref = ref.index_select(0, rows)
        elif kind == "wo":
            ref = ref[:, q0:q0 + tpm.q_dim]
        elif kind == "wgu":
            ref = ref[2 * f0:2 * (f0 + tpm.F)]
        elif kind == "wdown":
            ref = ref[:, f0:f0 + tpm.F]
        errs[name] = rel(tpm.g[name], ref)
    bad = {k: v for k, v in errs.items() if not v < 3e-2}
    assert not bad, ("pp x tp gradients", bad)
    # ---- 2. PPO-RLHF, PP x TP
    rcfg = RLHFConfig(model=LMConfig.tiny(n_layers=4), num_prompts=8, prompt_len=64, response_len=64,
                      micro_batch=2, lr=1e-4)
    tr = PPORLHFTrainer(rcfg, dev, tp=TP)
    w0 = tr.stage.model.flat.clone()
    for _ in range(2):
        out = tr.step()
        for k in ("pg_loss", "vf_loss", "kl", "reward_mean"):
            assert out[k] == out[k], (k, out)  # not NaN
    assert not torch.equal(w0, tr.stage.model.flat)
    tr.sync_weights()
    sm, rl = tr.stage.model, tr.rollout
    q0, f0 = sm.rank * sm.q_dim, sm.rank * sm.F
    for i in sm.layers:
        P = f"l{i}."
        assert torch.equal(rl.s[P + "wo"][:, q0:q0 + sm.q_dim], sm.s[P + "wo"]), P
        assert torch.equal(rl.s[P + "wgu"][2 * f0:2 * (f0 + sm.F)], sm.s[P + "wgu"]), P
        assert torch.equal(rl.s[P + "wdown"][:, f0:f0 + sm.F], sm.s[P + "wdown"]), P
        assert torch.equal(rl.s[P + "ln1"], sm.s[P + "ln1"]), P
    tr.tp_comm.check()
    if rank == 0:
        print("PP_TP_WORKER_OK", max(errs.values()), out)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
