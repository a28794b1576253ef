"""Tensor-parallel decoder forward (Megatron-style with sequence-parallel
activations) on the fused NVLink kernels of :mod:`turbol_b200.parallel.tp`.

Sharding over the ``tp`` ranks of a :class:`TensorParallelComm`:

* QKV projection: column-parallel by heads - rank r holds query heads
  [r*Hq/tp, (r+1)*Hq/tp) and KV heads [r*Hk/tp, (r+1)*Hk/tp) (rows of
  ``wqkv`` and ``bqkv`` in [q | k | v] order);
* output projection: row-parallel (the matching columns of ``wo``);
* gate/up projection: column-parallel over the interleaved (gate, up) row
  pairs; down projection: row-parallel (the matching columns of ``wdown``);
* embeddings, norms and the LM head: replicated.

Between blocks the residual stream is split by rows (tokens): rank r holds
rows [r*N/tp, (r+1)*N/tp).  Each column-parallel GEMM is an all-gather ->
GEMM kernel and each row-parallel GEMM a GEMM -> reduce-scatter kernel with
the residual add in its finishing pass, so a layer is

    h1 = rmsnorm(x_r);  qkv = AG-GEMM(h1, Wqkv_r) (+bias);  rope;  attention (local heads)
    x2_r = GEMM-RS(attn, Wo_r) + x_r;  h2 = rmsnorm(x2_r)
    act = AG-GEMM(h2, Wgu_r) with the SwiGLU epilogue;  x_r = GEMM-RS(act, Wdown_r) + x2_r

Row shards must be multiples of 128 rows (the GEMM's M tile).
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .._native import ops as _ops
from .llm import DecoderLM


class TPDecoderLM:
    def __init__(self, full: DecoderLM, comm):
        cfg = full.cfg
        tp, r = comm.world, comm.rank
        if cfg.n_heads % tp or cfg.n_kv_heads % tp or cfg.ffn % tp:
            raise ValueError("heads, KV heads and the FFN width must divide by the tensor-parallel size")
        self.cfg, self.comm, self.tp, self.rank = cfg, comm, tp, r
        self.device = full.device
        self.layers = list(full.layers)
        D = cfg.head_dim
        self.hq, self.hk = cfg.n_heads // tp, cfg.n_kv_heads // tp
        self.q_dim, self.kv_dim = self.hq * D, self.hk * D
        self.qkv_dim = self.q_dim + 2 * self.kv_dim
        self.F = cfg.ffn // tp
        self.table = full.table
        self.full = full  # replicated pieces: embedding, final norm, LM head
        self.w = {}
        self.load_from(full)

    @torch.no_grad()
    def load_from(self, full: DecoderLM):
        """(Re)slices this rank's shard out of a full model's bf16 weights (the
        trainer -> rollout weight sync when every rank holds the full model)."""
        cfg, r = self.cfg, self.rank
        Q, KV = cfg.q_dim, cfg.kv_dim
        q0, k0 = r * self.q_dim, r * self.kv_dim
        f0 = r * self.F
        def put(key, val):
            # in place once allocated: captured decode graphs keep these addresses
            if key in self.w:
                self.w[key].copy_(val)
            else:
                self.w[key] = val.contiguous().clone()

        rows = torch.cat([torch.arange(q0, q0 + self.q_dim), torch.arange(Q + k0, Q + k0 + self.kv_dim),
                          torch.arange(Q + KV + k0, Q + KV + k0 + self.kv_dim)]).to(self.device)
        for i in self.layers:
            P = f"l{i}."
            put(P + "wqkv", full.s[P + "wqkv"].index_select(0, rows))
            if cfg.qkv_bias:
                put(P + "bqkv", full.f32[P + "bqkv"].index_select(0, rows).float())
            put(P + "wo", full.s[P + "wo"][:, q0:q0 + self.q_dim])
            put(P + "wgu", full.s[P + "wgu"][2 * f0:2 * (f0 + self.F)])
            put(P + "wdown", full.s[P + "wdown"][:, f0:f0 + self.F])
            put(P + "ln1", full.f32[P + "ln1"].float())
            put(P + "ln2", full.f32[P + "ln2"].float())

    # ------------------------------------------------------------------ pieces
    def rows_of(self, n: int):
        if n % self.tp or (n // self.tp) % 128:
            raise ValueError(f"{n} rows: the per-rank share must be a multiple of 128")
        m = n // self.tp
        return self.rank * m, m

    def embed_rows(self, ids_flat: torch.Tensor) -> torch.Tensor:
        """This rank's rows of the embedding of ids_flat [N]."""
        r0, m = self.rows_of(ids_flat.numel())
        return self.full.embed(ids_flat[r0:r0 + m])

    def layer(self, i: int, x: torch.Tensor, pos_full: torch.Tensor, B: int, T: int, attn_fn, kv_hook=None):
        """One block on this rank's rows x [N/tp, H] -> [N/tp, H].  attn_fn(qkv,
        out) computes attention for the local heads over all N rows."""
        o, cfg, c = _ops(), self.cfg, self.comm
        P = f"l{i}."
        w = self.w
        N = x.shape[0] * self.tp
        h1 = torch.empty_like(x)
        o.rmsnorm_fwd(x, w[P + "ln1"], h1, None, cfg.rms_eps)
        if cfg.qkv_bias:
            qkv = c.all_gather_gemm(h1, w[P + "wqkv"], bias=w[P + "bqkv"], epi=o.EPI_BIAS)
        else:
            qkv = c.all_gather_gemm(h1, w[P + "wqkv"])
        o.rope(qkv, pos_full, self.table, self.hq + self.hk, cfg.head_dim)
        if kv_hook is not None:
            kv_hook(i, qkv)
        attn = torch.empty(N, self.q_dim, device=x.device, dtype=torch.bfloat16)
        attn_fn(qkv, attn)
        x2 = c.gemm_reduce_scatter(attn, w[P + "wo"], residual=x)
        h2 = torch.empty_like(x2)
        o.rmsnorm_fwd(x2, w[P + "ln2"], h2, None, cfg.rms_eps)
        act = c.all_gather_gemm(h2, w[P + "wgu"], epi=o.EPI_SWIGLU)
        return c.gemm_reduce_scatter(act, w[P + "wdown"], residual=x2)

    def forward(self, x: torch.Tensor, B: int, T: int, pos_full: torch.Tensor, kv_hook=None) -> torch.Tensor:
        """Full-sequence (prefill) forward of this rank's rows x [B*T/tp, H]."""
        o, cfg = _ops(), self.cfg
        scale = 1.0 / math.sqrt(cfg.head_dim)

        def attn_fn(qkv, out):
            q = qkv[:, : self.q_dim]
            k = qkv[:, self.q_dim:self.q_dim + self.kv_dim]
            v = qkv[:, self.q_dim + self.kv_dim:]
            o.flash_attn_fwd(q, k, v, out, None, B, T, self.hq, self.hk, scale)

        for i in self.layers:
            x = self.layer(i, x, pos_full, B, T, attn_fn, kv_hook)
        return x

    def final_norm(self, x: torch.Tensor) -> torch.Tensor:
        return self.full.final_norm(x)

    def logits(self, h: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.full.logits(h, out)
