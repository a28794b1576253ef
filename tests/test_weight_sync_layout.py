"""The trainer -> rollout weight sync's copy plan, checked on the CPU: running
every rank's segments of `TPReplicaSync` (what `tb_peer_scatter_copy` does
with peer stores) into every rank's replica buffer rebuilds the full model
on each rank, bf16 weights and fp32 norms / QKV bias alike."""
import math
import types

import pytest
import torch

from turbol_b200.models.llm import DecoderLM, LMConfig
from turbol_b200.models.tp_llm import TPTrainLM
from turbol_b200.parallel.weight_sync import TPReplicaSync, _align


def _fake_comm(world, rank):
    return types.SimpleNamespace(world=world, rank=rank, group=None)


def _run_segments(segs, src_bf16, src_f32, payloads, rank):
    """The scatter copy of one source rank: segment fields are
    (vec_begin, src_off, src_ld, dst_off, dst_ld, rows, row_bytes, src_sel, peers), in bytes."""
    srcs = (src_bf16.view(torch.uint8), src_f32.view(torch.uint8))
    for _, so, sl, do, dl, rows, rb, sel, peers in segs:
        assert rb % 16 == 0 and so % 16 == 0 and do % 16 == 0 and sl % 16 == 0 and dl % 16 == 0
        src = srcs[sel]
        for d in (range(len(payloads)) if peers else [rank]):
            for i in range(rows):
                payloads[d][do + i * dl:do + i * dl + rb] = src[so + i * sl:so + i * sl + rb]


@pytest.mark.parametrize("tie,bias", [(True, True), (False, False)])
def test_scatter_copy_plan_rebuilds_the_full_model_on_every_rank(tie, bias):
    cfg = LMConfig.tiny(n_layers=2)
    cfg.tie_embeddings, cfg.qkv_bias = tie, bias
    full = DecoderLM(cfg, "cpu", seed=5)
    tp = 2
    parts = [TPTrainLM(full, _fake_comm(tp, r)) for r in range(tp)]
    plans = []
    for p in parts:
        s = TPReplicaSync.__new__(TPReplicaSync)
        s._layout(p)
        plans.append((s, s._segments(cfg, p)))
    s0 = plans[0][0]
    size = s0.bf16_bytes + _align(s0.f32_numel * 4)
    payloads = [torch.zeros(size, dtype=torch.uint8) for _ in range(tp)]
    for r, (p, (_, segs)) in enumerate(zip(parts, plans)):
        _run_segments(segs, p.shadow, p.flat, payloads, r)
    for d in range(tp):
        bf = payloads[d][: s0.full_numel * 2].view(torch.bfloat16)
        f32 = payloads[d][s0.bf16_bytes:s0.bf16_bytes + s0.f32_numel * 4].view(torch.float32)
        for name, (off, shape) in s0.full_offsets.items():
            n = math.prod(shape)
            assert torch.equal(bf[off:off + n].view(shape), full.s[name]), (d, name)
        for name, (off, shape) in s0.f32_offsets.items():
            n = math.prod(shape)
            assert torch.equal(f32[off:off + n].view(shape), full.p[name]), (d, name)
    # what crosses NVLink: each rank's shard segments, once per peer
    sent = sum(s[5] * s[6] for s in plans[0][1] if s[8]) * (tp - 1)
    shard_bytes = sum(math.prod(sh) * 2 for n, (_, sh) in parts[0].offsets.items()
                      if n.endswith(("wqkv", "wo", "wgu", "wdown"))) + \
        sum(math.prod(sh) * 6 for n, (_, sh) in parts[0].offsets.items() if n.endswith("bqkv"))
    assert sent == shard_bytes * (tp - 1)
