"""Trainer -> rollout weight sync for a tensor-parallel trainer: a full-model
bf16 copy on every rank of the TP group, refreshed by one fused kernel.

At decode sizes a tensor-parallel rollout pays two cross-GPU collectives per
layer per token, each with a fixed latency far above the GEMMs they split;
a full copy per GPU decodes with no collective at all (each rank generates
its share of the group's sequences).  The copy has to follow every optimizer
step of the sharded trainer, which is an all-gather of the TP shards *and* a
layout change (QKV and gate/up shards are row blocks of the full matrices, O
and down shards are column blocks).  :class:`TPReplicaSync` does both in one
launch of ``tb_peer_scatter_copy`` (``csrc/kernels/comm.cu``): the replica
lives in NVLink-mapped peer memory (:class:`PeerBuffers`), and every rank
stores the rows of its shard segments straight into every rank's replica at
their full-model positions (16-byte peer stores), while the replicated
tensors (embedding, norms) are copied into the local replica only.  No NCCL
call, no staging buffer, no second local copy; the kernel's flag handshakes
order it against the readers of the replica on every rank.

The replica is a bf16-only :class:`DecoderLM` whose fp32 norm weights and QKV
bias (what the kernels read in fp32) sit in a second region of the same peer
buffer and are filled from the trainer's fp32 master weights.

Roofline: each rank sends (tp - 1) x its shard bytes over NVLink; at the
measured 770 GB/s per direction that is the floor for one sync.
"""
from __future__ import annotations

import math
from typing import List

import torch

from ..models.llm import ALIGN, DecoderLM
from .peer import PeerBuffers

_F32_NAMES = ("ln1", "ln2", "norm", "bqkv")


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


class TPReplicaSync:
    def __init__(self, model, group=None):
        """model: this rank's :class:`TPTrainLM` (master weights required)."""
        if model.flat is None:
            raise ValueError("TPReplicaSync needs the trainer's fp32 master weights")
        self.model = model
        cfg = model.cfg
        dev = model.device
        self._layout(model)
        self.pb = PeerBuffers(self.bf16_bytes + _align(self.f32_numel * 4), group, device=dev.index)
        shadow = self.pb.tensor(0, self.full_numel, torch.bfloat16)
        self.full = DecoderLM(cfg, dev, layers=model.layers, embed=model.has_embed, head=model.has_head,
                              master=False, storage={"flat": None, "grad": None, "shadow": shadow})
        if self.full.offsets != self.full_offsets or self.full.numel != self.full_numel:
            raise RuntimeError("weight sync: replica layout differs from DecoderLM's")
        f32 = self.pb.tensor(self.bf16_bytes, max(self.f32_numel, 1), torch.float32)
        self.full.f32 = {n: f32[o:o + math.prod(s)].view(s) for n, (o, s) in self.f32_offsets.items()}
        segs = self._segments(cfg, model)
        self.total_vecs = int(segs[-1][0] + segs[-1][5] * segs[-1][6] // 16) if segs else 0
        t = torch.tensor([[s[0], s[1], s[2], s[3], s[4], s[5], s[6], (s[7] & 0xFFFFFFFF) | (s[8] << 32)]
                          for s in segs], dtype=torch.int64)
        self.segs = t.to(dev)
        self.n_seg = len(segs)
        self.bytes_sent = sum(s[5] * s[6] for s in segs if s[8]) * (self.tp - 1)

    def _layout(self, model):
        """Offsets of the full replica (bf16) and of its fp32 tensors in the
        peer buffer: [bf16 replica | fp32 norms and QKV bias]."""
        self.tp, self.rank = model.tp, model.rank
        self.full_offsets, self.full_numel = self._full_layout(model.cfg, model)
        self.f32_offsets, off = {}, 0
        for name, (_, shape) in self.full_offsets.items():
            if name.endswith(_F32_NAMES):
                self.f32_offsets[name] = (off, shape)
                off += (math.prod(shape) + ALIGN - 1) // ALIGN * ALIGN
        self.f32_numel = off
        self.bf16_bytes = _align(self.full_numel * 2)

    @staticmethod
    def _full_layout(cfg, model):
        """Offsets of a full DecoderLM holding the same layers / embedding / head."""
        offsets, off = {}, 0
        H, F = cfg.hidden, cfg.ffn

        def add(name, shape):
            nonlocal off
            offsets[name] = (off, tuple(shape))
            off += (math.prod(shape) + ALIGN - 1) // ALIGN * ALIGN

        if model.has_embed or (model.has_head and cfg.tie_embeddings):
            add("embed", (cfg.vocab, H))
        for i in model.layers:
            add(f"l{i}.ln1", (H,))
            add(f"l{i}.wqkv", (cfg.qkv_dim, H))
            if cfg.qkv_bias:
                add(f"l{i}.bqkv", (cfg.qkv_dim,))
            add(f"l{i}.wo", (H, cfg.q_dim))
            add(f"l{i}.ln2", (H,))
            add(f"l{i}.wgu", (2 * F, H))
            add(f"l{i}.wdown", (H, F))
        if model.has_head:
            add("norm", (H,))
            if not cfg.tie_embeddings:
                add("lm_head", (cfg.vocab, H))
        return offsets, off

    def _segments(self, cfg, model) -> List[tuple]:
        """(vec_begin, src_off, src_ld, dst_off, dst_ld, rows, row_bytes, src_sel, peers) in bytes."""
        tp, r = self.tp, self.rank
        D = cfg.head_dim
        qd, kd, F = cfg.n_heads // tp * D, cfg.n_kv_heads // tp * D, cfg.ffn // tp
        Q, KV, H, FF = cfg.q_dim, cfg.kv_dim, cfg.hidden, cfg.ffn
        q0, k0, f0 = r * qd, r * kd, r * F
        out = []

        def seg(sel, s_el, d_el, rows, row_el, s_ld_el, d_ld_el, peers, es):
            # sel 0: bf16 shadow -> bf16 replica; sel 1: fp32 master -> fp32 region
            base = 0 if sel == 0 else self.bf16_bytes
            rb, sl, dl = row_el * es, s_ld_el * es, d_ld_el * es
            so, do = s_el * es, base + d_el * es
            for v, what in ((rb, "row bytes"), (sl, "source stride"), (dl, "replica stride"), (so, "source offset"),
                            (do, "replica offset")):
                if v % 16:
                    raise ValueError(f"weight sync: {what} {v} is not a multiple of 16 bytes")
            out.append([0, so, sl, do, dl, rows, rb, sel, 1 if peers else 0])

        for name, (soff, sshape) in model.offsets.items():
            if name not in self.full_offsets:
                continue
            doff, dshape = self.full_offsets[name]
            kind = name.rsplit(".", 1)[-1]
            passes = [(0, 2, doff)]
            if name in self.f32_offsets:
                passes.append((1, 4, self.f32_offsets[name][0]))
            for sel, es, dbase in passes:
                if kind == "wqkv":  # row blocks: this rank's q, k and v heads
                    seg(sel, soff, dbase + q0 * H, qd, H, H, H, True, es)
                    seg(sel, soff + qd * H, dbase + (Q + k0) * H, kd, H, H, H, True, es)
                    seg(sel, soff + (qd + kd) * H, dbase + (Q + KV + k0) * H, kd, H, H, H, True, es)
                elif kind == "bqkv":
                    seg(sel, soff, dbase + q0, 1, qd, qd, qd, True, es)
                    seg(sel, soff + qd, dbase + Q + k0, 1, kd, kd, kd, True, es)
                    seg(sel, soff + qd + kd, dbase + Q + KV + k0, 1, kd, kd, kd, True, es)
                elif kind == "wo":
                    seg(sel, soff, dbase + q0, H, qd, qd, Q, True, es)
                elif kind == "wgu":
                    seg(sel, soff, dbase + 2 * f0 * H, 2 * F, H, H, H, True, es)
                elif kind == "wdown":
                    seg(sel, soff, dbase + f0, H, F, F, FF, True, es)
                else:  # replicated: every rank holds the same values, copy into the local replica only
                    n = math.prod(sshape)
                    seg(sel, soff, dbase, 1, n, n, n, False, es)
        vb = 0
        for s in out:
            s[0] = vb
            vb += s[5] * s[6] // 16
        return [tuple(s) for s in out]

    @torch.no_grad()
    def __call__(self):
        """Refreshes every rank's replica from the trainer shards (all ranks of
        the group call it, in the same order as their other collectives)."""
        if self.n_seg == 0:
            return
        m = self.model
        self.pb.mem.scatter_copy(m.shadow, m.flat, self.segs, self.total_vecs, 0)

    def check(self):
        self.pb.check()
