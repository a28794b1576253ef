"""Worker for the tensor-parallel training test (2 GPUs, torchrun).

1. TPTrainLM forward (save) + backward on the fused all-gather->GEMM /
   GEMM->reduce-scatter kernels matches the single-GPU DecoderLM forward and
   hand-written backward: outputs and input gradients on each rank's rows,
   the sharded weight gradients against the matching slices of the full
   gradients, the replicated ones (norms, embedding) after the TP all-reduce.
2. The fused trainer -> rollout weight sync (TPReplicaSync): every rank's
   full-model replica equals the source model, and after the shards move it
   equals the un-sharded shards of both ranks (bit for bit).
3. GRPO with tensor-parallel training (tp=2, tp_mode="train") runs two steps
   with the full-replica rollout and with the TP rollout: finite statistics,
   replicated weights stay identical on both ranks, the shards move, and the
   replica follows the trainer."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200.models.llm import DecoderLM, LMConfig  # noqa: E402
from turbol_b200.models.tp_llm import TPTrainLM  # noqa: E402
from turbol_b200.parallel.tp import TensorParallelComm  # noqa: E402
from turbol_b200.rl.grpo import GRPOConfig, GRPOTrainer  # noqa: E402


def rel(a, b):
    a, b = a.float(), b.float()
    return (a - b).abs().max().item() / (b.abs().max().item() + 1e-6)


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = LMConfig.tiny(n_layers=2)
    cfg.init_std = 0.05
    full = DecoderLM(cfg, dev, seed=3)
    comm = TensorParallelComm(max_rows=2048, max_in=cfg.hidden, max_out=cfg.hidden)
    tpm = TPTrainLM(full, comm)
    B, T = 4, 128
    N, m = B * T, B * T // world
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.vocab, (B, T), generator=g).to(dev, torch.int32)
    dy = (torch.randn(N, cfg.hidden, generator=g) * 0.1).to(dev, torch.bfloat16)
    pos = torch.arange(T, device=dev, dtype=torch.int32).repeat(B)
    # ---- single-GPU reference
    full.zero_grad()
    y_ref, saved = full.forward(full.embed(ids), B, T, pos, save=True)
    dx_ref = full.backward(dy, saved, B, T, pos)
    full.embed_backward(ids, dx_ref)
    # ---- tensor parallel (twice: the second call runs on the other parity of the staging buffers)
    r0 = rank * m
    for rep in range(2):
        tpm.zero_grad()
        x = tpm.embed_rows(ids.reshape(-1))
        y, sv = tpm.forward_train(x, B, T, pos, save=True)
        dx = tpm.backward(dy[r0:r0 + m].contiguous(), sv, B, T, pos)
        tpm.embed_backward_rows(ids.reshape(-1), dx)
        tpm.reduce_replicated_grads()
        torch.cuda.synchronize()
        comm.check()
        errs = {"y": rel(y, y_ref[r0:r0 + m]), "dx": rel(dx, dx_ref[r0:r0 + m])}
        Q, KV, D = cfg.q_dim, cfg.kv_dim, cfg.head_dim
        q0, k0, f0 = rank * tpm.q_dim, rank * tpm.kv_dim, rank * tpm.F
        rows = torch.cat([torch.arange(q0, q0 + tpm.q_dim), torch.arange(Q + k0, Q + k0 + tpm.kv_dim),
                          torch.arange(Q + KV + k0, Q + KV + k0 + tpm.kv_dim)]).to(dev)
        for i in tpm.layers:
            P = f"l{i}."
            errs[P + "wqkv"] = rel(tpm.g[P + "wqkv"], full.g[P + "wqkv"].index_select(0, rows))
            errs[P + "bqkv"] = rel(tpm.g[P + "bqkv"], full.g[P + "bqkv"].index_select(0, rows))
            errs[P + "wo"] = rel(tpm.g[P + "wo"], full.g[P + "wo"][:, q0:q0 + tpm.q_dim])
            errs[P + "wgu"] = rel(tpm.g[P + "wgu"], full.g[P + "wgu"][2 * f0:2 * (f0 + tpm.F)])
            errs[P + "wdown"] = rel(tpm.g[P + "wdown"], full.g[P + "wdown"][:, f0:f0 + tpm.F])
            errs[P + "ln1"] = rel(tpm.g[P + "ln1"], full.g[P + "ln1"])
            errs[P + "ln2"] = rel(tpm.g[P + "ln2"], full.g[P + "ln2"])
        errs["embed"] = rel(tpm.g["embed"], full.g["embed"])
        bad = {k: v for k, v in errs.items() if not v < 3e-2}
        assert not bad, ("tp train", rep, bad)
    # ---- fused trainer -> rollout weight sync: the full replica on every rank
    from turbol_b200.parallel.weight_sync import TPReplicaSync

    sync = TPReplicaSync(tpm)
    sync()
    torch.cuda.synchronize()
    sync.check()
    for name in full.offsets:
        assert torch.equal(sync.full.s[name], full.s[name]), ("replica bf16", name)
    for name, t in sync.full.f32.items():
        assert torch.equal(t, full.p[name]), ("replica fp32", name)
    with torch.no_grad():  # move the shards (rank-dependent), sync, compare with the un-sharded shards
        tpm.flat.add_(torch.randn(tpm.numel, generator=torch.Generator(device=dev).manual_seed(7 + rank),
                                  device=dev) * 1e-2)
        rep = tpm.flat[: tpm.rep_numel].clone()
        dist.broadcast(rep, src=0)  # replicated tensors stay identical across the group
        tpm.flat[: tpm.rep_numel].copy_(rep)
        tpm.shadow.copy_(tpm.flat)
    sync()
    torch.cuda.synchronize()
    sync.check()
    flats = [torch.empty_like(tpm.flat) for _ in range(world)]
    dist.all_gather(flats, tpm.flat)
    want = DecoderLM(cfg, dev, seed=3)
    for t, f in enumerate(flats):
        TPTrainLM.unshard_into(want, f, tpm.offsets, world, t, shards_only=t > 0)
    want.sync_shadow()
    for name in full.offsets:
        assert torch.equal(sync.full.s[name], want.s[name]), ("replica after sync", name)
    for name, t in sync.full.f32.items():
        assert torch.equal(t, want.p[name]), ("replica fp32 after sync", name)
    # ---- GRPO with tensor-parallel training: full-replica rollout (default) and TP rollout
    # (the TP decode step needs a multiple of 128 sequences per rank)
    gcfg = GRPOConfig(model=cfg, num_prompts=32, group_size=8, prompt_len=64, response_len=64, micro_batch=8,
                      lr=1e-3)
    for mode in ("replica", "tp"):
        tr = GRPOTrainer(gcfg, str(dev), dp="fused", tp=2, tp_mode="train", rollout=mode)
        before = tr.model.flat.clone()
        for _ in range(2):
            st = tr.step()
            assert all(v == v for v in st.values() if isinstance(v, float)), (mode, st)
        torch.cuda.synchronize()
        tr.comm.check()
        if tr.sync is not None:
            tr.sync.check()
            # the replica holds the trainer's latest weights
            flats = [torch.empty_like(tr.model.flat) for _ in range(world)]
            dist.all_gather(flats, tr.model.flat)
            chk = DecoderLM(cfg, dev, seed=3)
            for t, f in enumerate(flats):
                TPTrainLM.unshard_into(chk, f, tr.model.offsets, world, t, shards_only=t > 0)
            chk.sync_shadow()
            for name in chk.offsets:
                assert torch.equal(tr.sync.full.s[name], chk.s[name]), ("GRPO replica", name)
        moved = (tr.model.flat - before).abs().max().item()
        assert moved > 0, "weights did not move"
        if mode == "replica":
            # sharded checkpoint: every rank writes its own TP shard and marker, and a
            # fresh trainer on each rank gets its own shard back bit for bit
            import tempfile

            from turbol_b200.utils.checkpoint import latest_step, load_checkpoint, save_checkpoint

            base = os.path.join(tempfile.gettempdir(), f"tb_tp_ckpt_{os.environ.get('MASTER_PORT', '0')}")
            save_checkpoint(base, 2, tr)
            dist.barrier()
            names = set(os.listdir(os.path.join(base, "step_2")))
            want = {f"policy_tp{t}_pp0.pt" for t in range(world)} | {f"COMPLETE_dp0_tp{t}_pp0" for t in range(world)}
            assert want <= names and latest_step(base) == 2, names
            tr2 = GRPOTrainer(gcfg, str(dev), dp="fused", tp=2, tp_mode="train", rollout=mode)
            load_checkpoint(base, trainer=tr2)
            torch.cuda.synchronize()
            assert torch.equal(tr2.model.flat, tr.model.flat) and tr2.step_count == tr.step_count
            for name in chk.offsets:  # the replica follows the loaded shards
                assert torch.equal(tr2.sync.full.s[name], chk.s[name]), ("replica after load", name)
            dist.barrier()
            if rank == 0:
                import shutil

                shutil.rmtree(base, ignore_errors=True)
            del tr2
        rep_sum = tr.model.flat[: tr.model.rep_numel].double().sum().reshape(1)
        sums = [torch.zeros_like(rep_sum) for _ in range(world)]
        dist.all_gather(sums, rep_sum)
        assert float(sums[0]) == float(sums[1]), ("replicated weights diverged", [float(s) for s in sums])
        del tr
    if rank == 0:
        print("TP_TRAIN_WORKER_OK", {k: round(v, 5) for k, v in errs.items()}, st["kl"], moved)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
