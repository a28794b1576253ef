"""Tensor-parallel training layout on the CPU: the shards of every rank put
back together give the full model, replicated parameters come first, and the
GRPO trainer's row ownership covers every sequence once."""
import types

import pytest
import torch

from turbol_b200.models.llm import DecoderLM, LMConfig
from turbol_b200.models.tp_llm import TPTrainLM


def _fake_comm(world, rank):
    return types.SimpleNamespace(world=world, rank=rank, group=None)


@pytest.mark.parametrize("tie", [True, False])
def test_shards_reassemble_full_model(tie):
    cfg = LMConfig.tiny(n_layers=2)
    cfg.tie_embeddings = tie
    cfg.qkv_bias = tie
    full = DecoderLM(cfg, "cpu", seed=1)
    tp = 2
    parts = [TPTrainLM(full, _fake_comm(tp, r)) for r in range(tp)]
    for p in parts:
        # replicated first, then shards; the fp32 master and the bf16 copy agree
        assert max(o for o, _ in (p.offsets[n] for n in p.offsets if n.endswith(("ln1", "ln2", "norm")))) < \
            p.rep_numel <= min(o for o, _ in (p.offsets[n] for n in p.offsets if n.endswith("wqkv")))
        assert torch.equal(p.shadow, p.flat.to(torch.bfloat16))
        assert torch.equal(p.p["embed"], full.p["embed"])
    Q, KV = cfg.q_dim, cfg.kv_dim
    for i in range(cfg.n_layers):
        P = f"l{i}."
        q = torch.cat([p.p[P + "wqkv"][: p.q_dim] for p in parts])
        k = torch.cat([p.p[P + "wqkv"][p.q_dim:p.q_dim + p.kv_dim] for p in parts])
        v = torch.cat([p.p[P + "wqkv"][p.q_dim + p.kv_dim:] for p in parts])
        assert torch.equal(torch.cat([q, k, v]), full.p[P + "wqkv"])
        assert torch.equal(torch.cat([p.p[P + "wo"] for p in parts], 1), full.p[P + "wo"])
        assert torch.equal(torch.cat([p.p[P + "wgu"] for p in parts]), full.p[P + "wgu"])
        assert torch.equal(torch.cat([p.p[P + "wdown"] for p in parts], 1), full.p[P + "wdown"])
        if cfg.qkv_bias:
            b = full.p[P + "bqkv"]
            got = torch.cat([torch.cat([p.p[P + "bqkv"][: p.q_dim] for p in parts]),
                             torch.cat([p.p[P + "bqkv"][p.q_dim:p.q_dim + p.kv_dim] for p in parts]),
                             torch.cat([p.p[P + "bqkv"][p.q_dim + p.kv_dim:] for p in parts])])
            assert torch.equal(got, b)
    # a frozen copy holds the same bf16 weights and no master / gradient
    fz = parts[1].frozen_copy()
    assert fz.flat is None and fz.grad is None and torch.equal(fz.shadow, parts[1].shadow)
    assert torch.equal(fz.f32["l0.ln1"], parts[1].p["l0.ln1"])


def test_shard_sizes_and_validation():
    cfg = LMConfig.tiny(n_layers=1)
    full = DecoderLM(cfg, "cpu", seed=0)
    p = TPTrainLM(full, _fake_comm(2, 0))
    H, D = cfg.hidden, cfg.head_dim
    per = (cfg.n_heads // 2 + cfg.n_kv_heads) * D * H + (cfg.n_heads // 2 + cfg.n_kv_heads) * D \
        + H * (cfg.n_heads // 2) * D + 3 * (cfg.ffn // 2) * H
    shard_numel = sum(torch.Size(s).numel() for n, (_, s) in p.offsets.items() if not n.endswith(
        ("ln1", "ln2", "norm", "embed", "lm_head")))
    assert shard_numel == per
    with pytest.raises(ValueError):
        TPTrainLM(full, _fake_comm(3, 0))  # 4 heads do not split over 3 ranks


def test_grpo_row_ownership_covers_batch():
    from turbol_b200.rl.grpo import GRPOTrainer

    owned = []
    for r in range(2):
        t = GRPOTrainer.__new__(GRPOTrainer)
        t.cfg = types.SimpleNamespace(micro_batch=8)
        t.tp, t.tp_rank, t.device = 2, r, torch.device("cpu")
        owned.append(t._tp_own(32))
    allv = torch.cat(owned).sort().values
    assert torch.equal(allv, torch.arange(32))
    assert owned[0][:4].tolist() == [0, 1, 2, 3] and owned[1][:4].tolist() == [4, 5, 6, 7]


@pytest.mark.parametrize("master", [True, False])
def test_unshard_inverts_load(master):
    """Writing every rank's shard back into an empty full model rebuilds it."""
    cfg = LMConfig.tiny(n_layers=2)
    src = DecoderLM(cfg, "cpu", seed=4)
    tp = 2
    dst = DecoderLM(cfg, "cpu", seed=9, master=master)
    for r in range(tp):
        part = TPTrainLM(src, _fake_comm(tp, r))
        buf = part.flat if master else part.shadow
        TPTrainLM.unshard_into(dst, buf, part.offsets, tp, r, shards_only=r > 0)
    ref = src.p if master else src.s
    got = dst.p if master else dst.s
    for n in src.offsets:
        assert torch.equal(got[n], ref[n].to(got[n].dtype)), n
    for n in dst.f32:
        assert torch.allclose(dst.f32[n], src.p[n], atol=1e-2), n


def test_grpo_tp_rejects_shapes_the_fused_kernels_cannot_tile(tmp_path):
    """Tensor-parallel GRPO checks its row counts before building anything."""
    import torch.distributed as dist

    from turbol_b200.rl.grpo import GRPOConfig, GRPOTrainer

    own = not dist.is_initialized()
    if own:
        dist.init_process_group("gloo", init_method=f"file://{tmp_path}/pg", rank=0, world_size=1)
    try:
        cfg = GRPOConfig(model=LMConfig.tiny(), num_prompts=4, group_size=2, prompt_len=64, response_len=64,
                         micro_batch=2)
        with pytest.raises(ValueError, match="multiple of 128"):
            GRPOTrainer(cfg, "cpu", dp="nccl", tp=2)
    finally:
        if own:
            dist.destroy_process_group()
