"""Worker for the pipeline-parallel tests (2 GPUs, torchrun).
1. A 2-stage 1F1B pass gives the same weight gradients as the whole model on
   one GPU (loss: sum of the targets' log-probs over 4 micro-batches).
2. PPO-RLHF on a tiny policy with a value head runs through the pipeline;
   the rollout copy equals the stages' weights after the weight sync."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200._native import ops  # noqa: E402
from turbol_b200.models.llm import DecoderLM, LMConfig  # noqa: E402
from turbol_b200.parallel import pipeline as pp  # noqa: E402
from turbol_b200.rl.ppo_rlhf import PPORLHFTrainer, RLHFConfig  # noqa: E402


def grads_full(full, ids, mb, T):
    o = ops()
    pos = torch.arange(T, device=ids.device, dtype=torch.int32).repeat(mb)
    full.zero_grad()
    for i in range(ids.shape[0] // mb):
        x_ids = ids[i * mb:(i + 1) * mb]
        x, saved = full.forward(full.embed(x_ids), mb, T, pos, save=True)
        dx = head_loss_grad(full, x, x_ids)
        dx = full.backward(dx, saved, mb, T, pos)
        full.embed_backward(x_ids, dx)


def head_loss_grad(model, x, ids):
    """d(sum of log p(next token)) / d x for every position but the last."""
    o = ops()
    N = x.shape[0]
    rstd = torch.empty(N, device=x.device)
    hf = model.final_norm(x, rstd)
    logits = model.logits(hf)
    tgt = torch.roll(ids.reshape(-1), -1).contiguous()
    dlp = torch.full((N,), -1e-3, device=x.device)
    o.logprob(logits, tgt, None, dlp)
    dh = torch.empty_like(hf)
    o.gemm(logits, model.head_weight(), dh, False, True)
    o.gemm(logits, hf, model.head_grad(), True, True, accumulate=True, split_k=1)
    dx = torch.empty_like(x)
    o.rmsnorm_bwd(dh, x, model.f32["norm"], rstd, dx, None, model.g["norm"])
    return dx


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = LMConfig.tiny(n_layers=4)
    cfg.tie_embeddings = False
    cfg.init_std = 0.05
    # ---- 1. pipeline gradients == single-GPU gradients
    full = DecoderLM(cfg, dev, seed=5)
    st = pp.PipelineStage(cfg, rank, world, dev)
    st.load_from_full(full)
    mb, T, M = 2, 64, 4
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, cfg.vocab, (mb * M, T), generator=g).to(dev, torch.int32)
    grads_full(full, ids, mb, T)
    pos = torch.arange(T, device=dev, dtype=torch.int32).repeat(mb)
    pp.set_micro_geometry(mb, T, pos)
    st.zero_grad()
    pp.run_1f1b(st, list(range(world)), M, mb * T,
                lambda i: st.model.embed(ids[i * mb:(i + 1) * mb]),
                lambda i, x: head_loss_grad(st.model, x, ids[i * mb:(i + 1) * mb]),
                lambda i, dx: st.model.embed_backward(ids[i * mb:(i + 1) * mb], dx))
    torch.cuda.synchronize()
    worst = 0.0
    for name in st.model.offsets:
        a, b = st.model.g[name], full.g[name]
        err = (a - b).abs().max().item() / (b.abs().max().item() + 1e-12)
        worst = max(worst, err)
    assert worst < 1e-4, ("pipeline gradients", worst)
    # ---- 1b. activation recompute: the same gradients
    ref_g = st.model.grad.clone()
    st.zero_grad()
    pp.run_1f1b(st, list(range(world)), M, mb * T,
                lambda i: st.model.embed(ids[i * mb:(i + 1) * mb]),
                lambda i, x: head_loss_grad(st.model, x, ids[i * mb:(i + 1) * mb]),
                lambda i, dx: st.model.embed_backward(ids[i * mb:(i + 1) * mb], dx), recompute=True)
    torch.cuda.synchronize()
    rel = (st.model.grad - ref_g).abs().max().item() / (ref_g.abs().max().item() + 1e-12)
    assert rel < 1e-5, ("recompute gradients", rel)
    # ---- 2. PPO-RLHF through the pipeline
    rcfg = RLHFConfig(model=LMConfig.tiny(n_layers=4), num_prompts=8, prompt_len=32, response_len=32,
                      micro_batch=2, lr=1e-4)
    tr = PPORLHFTrainer(rcfg, dev)
    w0 = tr.stage.model.flat.clone()
    for _ in range(2):
        out = tr.step()
        for k in ("pg_loss", "vf_loss", "kl", "reward_mean"):
            assert out[k] == out[k], (k, out)  # not NaN
    assert not torch.equal(w0, tr.stage.model.flat)
    tr.sync_weights()
    for name in tr._stage_names(rank):
        assert torch.equal(tr.rollout.s[name], tr.stage.model.s[name]), name
    # ---- 3. checkpoint of the pipeline shards: each stage saves policy_tp0_pp<s>, a fresh trainer loads it
    import tempfile

    from turbol_b200.utils.checkpoint import load_checkpoint, save_checkpoint

    base = os.path.join(tempfile.gettempdir(), f"tb_pp_ckpt_{os.environ.get('MASTER_PORT', '0')}")
    save_checkpoint(base, 3, tr)
    dist.barrier()
    names = set(os.listdir(os.path.join(base, "step_3")))
    assert {f"policy_tp0_pp{p}.pt" for p in range(world)} <= names, names
    tr2 = PPORLHFTrainer(rcfg, dev)
    load_checkpoint(base, trainer=tr2)
    torch.cuda.synchronize()
    assert torch.equal(tr2.stage.model.flat, tr.stage.model.flat) and tr2.step_count == tr.step_count
    for name in tr._stage_names(rank):
        assert torch.equal(tr2.rollout.s[name], tr.stage.model.s[name]), ("rollout after load", name)
    dist.barrier()
    if rank == 0:
        import shutil

        shutil.rmtree(base, ignore_errors=True)
    if rank == 0:
        print("PP_WORKER_OK", worst, out)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
