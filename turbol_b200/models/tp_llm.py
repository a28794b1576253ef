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

:class:`TPTrainLM` is the trainable variant: it owns this rank's shard as flat
fp32 master / fp32 gradient / bf16 buffers (replicated parameters first, so
their partial gradients are one contiguous all-reduce over the TP group) and
has a hand-written backward built from the same fused kernels:

    d act  = AG-GEMM(dx_r, Wdown_r)          (MN-major B; the gathered dX is kept for dWdown)
    d h2_r = GEMM-RS(d gu, Wgu_r)             (dWgu from the gathered h2 saved in forward)
    d attn = AG-GEMM(dx2_r, Wo_r)             (gathered dX2 for dWo)
    d h1_r = GEMM-RS(d qkv, Wqkv_r)           (dWqkv from the gathered h1)

Forward with ``save=True`` asks each all-gather GEMM for its gathered input
(the kernel writes it at the end of the same launch), so a training step moves
every activation row over NVLink once per direction and calls no NCCL
collective inside a layer.  The rollout engine can run on the same object
(``TPLLMGenerator``): the optimizer writes the bf16 weights it reads, so the
trainer -> rollout weight sync needs no copy at all.

Reference parity: the reference names tensor parallelism only in its
specification (docs/SPECIFICATION.md:1890-1900, a TENSOR_PARALLEL strategy and
a tensor_parallel_size field) and forwards tensor_parallel_size to vLLM
(turbol_vllm/python/turbol/vllm_inference.py:98,176); it has no tensor-parallel
model or training code.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .._native import ops as _ops
from .llm import ALIGN, DecoderLM


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

    def final_norm(self, x: torch.Tensor, rstd: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.full.final_norm(x, rstd)

    def logits(self, h: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.full.logits(h, out)


class _Replicated:
    """The replicated pieces of a :class:`TPTrainLM` (embedding, final norm, LM
    head) with the methods of :class:`DecoderLM` that read them."""

    embed = DecoderLM.embed
    final_norm = DecoderLM.final_norm
    logits = DecoderLM.logits
    head_weight = DecoderLM.head_weight
    head_grad = DecoderLM.head_grad

    def __init__(self, owner: "TPTrainLM"):
        self.owner = owner

    @property
    def cfg(self):
        return self.owner.cfg

    @property
    def device(self):
        return self.owner.device

    @property
    def s(self):
        return self.owner.s

    @property
    def f32(self):
        return self.owner.f32

    @property
    def g(self):
        return self.owner.g


class TPTrainLM(TPDecoderLM):
    """Tensor-parallel decoder that owns and trains its shard (see the module
    docstring).  ``master=False`` keeps only bf16 weights (a frozen reference
    copy for a KL penalty)."""

    def __init__(self, full: DecoderLM, comm, master: bool = True, storage: Optional[dict] = None):
        cfg = full.cfg
        tp, r = comm.world, comm.rank
        if cfg.n_heads % tp or cfg.n_kv_heads % tp or cfg.ffn % tp:
            raise ValueError("heads, KV heads and the FFN width must divide by the tensor-parallel size")
        self.has_embed, self.has_head = full.has_embed, full.has_head
        self.cfg, self.comm, self.tp, self.rank = cfg, comm, tp, r
        self.device = full.device
        self.layers = list(full.layers)
        D = cfg.head_dim
        self.hq, self.hk = cfg.n_heads // tp, cfg.n_kv_heads // tp
        self.q_dim, self.kv_dim = self.hq * D, self.hk * D
        self.qkv_dim = self.q_dim + 2 * self.kv_dim
        self.F = cfg.ffn // tp
        self.table = full.table
        self.has_master = master
        self.offsets, self.rep_numel, self.numel = self.layout(cfg, self.layers, self.has_embed, self.has_head, tp)
        off = self.numel
        if storage is not None:
            self.flat, self.grad, self.shadow = storage["flat"], storage["grad"], storage["shadow"]
        else:
            self.shadow = torch.zeros(off, device=self.device, dtype=torch.bfloat16)
            self.flat = torch.zeros(off, device=self.device) if master else None
            self.grad = torch.zeros(off, device=self.device) if master else None
        self._make_views()
        self.full = _Replicated(self)
        self._ws = {}
        if storage is None:
            self.load_from(full)

    @staticmethod
    def layout(cfg, layers, has_embed: bool, has_head: bool, tp: int):
        """(offsets {name: (offset, shape)}, replicated numel, numel) of one
        rank's flat buffers; the same on every rank of a TP group."""
        H, D = cfg.hidden, cfg.head_dim
        q_dim, kv_dim = cfg.n_heads // tp * D, cfg.n_kv_heads // tp * D
        qkv_dim, F = q_dim + 2 * kv_dim, cfg.ffn // tp
        offsets = {}
        off = 0

        def add(name, shape):
            nonlocal off
            offsets[name] = (off, tuple(shape))
            off += (math.prod(shape) + ALIGN - 1) // ALIGN * ALIGN

        # replicated (partial gradients, summed over the TP group) ...
        if has_embed or (has_head and cfg.tie_embeddings):
            add("embed", (cfg.vocab, H))
        if has_head:
            add("norm", (H,))
            if not cfg.tie_embeddings:
                add("lm_head", (cfg.vocab, H))
        for i in layers:
            add(f"l{i}.ln1", (H,))
            add(f"l{i}.ln2", (H,))
        rep = off
        # ... then this rank's shards (complete gradients)
        for i in layers:
            add(f"l{i}.wqkv", (qkv_dim, H))
            if cfg.qkv_bias:
                add(f"l{i}.bqkv", (qkv_dim,))
            add(f"l{i}.wo", (H, q_dim))
            add(f"l{i}.wgu", (2 * F, H))
            add(f"l{i}.wdown", (H, F))
        return offsets, rep, off

    @staticmethod
    @torch.no_grad()
    def unshard_into(full: DecoderLM, flat: torch.Tensor, offsets: dict, tp: int, rank: int, shards_only: bool = False):
        """Writes a TP rank's flat buffer (``flat`` laid out by ``offsets``) into
        the matching parts of a full model's weights: the shards into their
        slices, the replicated tensors whole (skipped with ``shards_only``).
        The inverse of :meth:`load_from`; the trainer -> rollout weight sync of
        a tensor-parallel trainer and a full-model rollout engine."""
        cfg = full.cfg
        D = cfg.head_dim
        qd, kd, F = cfg.n_heads // tp * D, cfg.n_kv_heads // tp * D, cfg.ffn // tp
        Q, KV = cfg.q_dim, cfg.kv_dim
        q0, k0, f0 = rank * qd, rank * kd, rank * F
        dst = full.p if full.flat is not None else full.s

        def view(name):
            o, shp = offsets[name]
            return flat[o:o + math.prod(shp)].view(shp)

        for name in offsets:
            if name not in full.offsets:
                continue
            v = view(name)
            kind = name.rsplit(".", 1)[-1]
            # the weights, and the separate fp32 copy a bf16-only model keeps of norms and biases
            tgts = [dst[name]] + ([full.f32[name]] if name in full.f32 and full.f32[name] is not dst[name] else [])
            for t in tgts:
                if kind in ("wqkv", "bqkv"):
                    t[q0:q0 + qd].copy_(v[:qd])
                    t[Q + k0:Q + k0 + kd].copy_(v[qd:qd + kd])
                    t[Q + KV + k0:Q + KV + k0 + kd].copy_(v[qd + kd:])
                elif kind == "wo":
                    t[:, q0:q0 + qd].copy_(v)
                elif kind == "wgu":
                    t[2 * f0:2 * (f0 + F)].copy_(v)
                elif kind == "wdown":
                    t[:, f0:f0 + F].copy_(v)
                elif not shards_only:
                    t.copy_(v)

    # ------------------------------------------------------------------ params
    def _make_views(self):
        def views(buf):
            if buf is None:
                return None
            return {n: buf[o:o + math.prod(s)].view(s) for n, (o, s) in self.offsets.items()}

        self.p, self.g, self.s = views(self.flat), views(self.grad), views(self.shadow)
        fp32 = ("ln1", "ln2", "norm", "bqkv")
        if self.flat is None:
            self.f32 = {n: self.s[n].float() for n in self.offsets if n.endswith(fp32)}
        else:
            self.f32 = self.p
        # what layer() reads: bf16 matrices, fp32 norms and biases
        self.w = {n: (self.f32[n] if n.endswith(fp32) else self.s[n]) for n in self.offsets}

    def rebind_storage(self, flat, grad, shadow):
        """Moves the weights into caller-provided flat buffers (e.g. the
        symmetric memory of a fused data-parallel optimizer)."""
        if flat is not None:
            flat[: self.numel].copy_(self.flat)
        shadow[: self.numel].copy_(self.shadow)
        if grad is not None:
            grad[: self.numel].zero_()
        self.flat = flat[: self.numel] if flat is not None else None
        self.grad = grad[: self.numel] if grad is not None else None
        self.shadow = shadow[: self.numel]
        self._make_views()

    @torch.no_grad()
    def load_from(self, full: DecoderLM):
        """Copies this rank's shard and the replicated parameters out of a full model."""
        cfg, r = self.cfg, self.rank
        Q, KV = cfg.q_dim, cfg.kv_dim
        q0, k0, f0 = r * self.q_dim, r * self.kv_dim, r * self.F
        src = full.p if full.flat is not None else full.s
        rows = torch.cat([torch.arange(q0, q0 + self.q_dim), torch.arange(Q + k0, Q + k0 + self.kv_dim),
                          torch.arange(Q + KV + k0, Q + KV + k0 + self.kv_dim)]).to(self.device)

        def put(name, val):
            if self.flat is not None:
                self.p[name].copy_(val)
            self.s[name].copy_(val)

        for name in ("embed", "lm_head"):
            if name in self.offsets:
                put(name, src[name])
        if "norm" in self.offsets:
            put("norm", full.f32["norm"])
        for i in self.layers:
            P = f"l{i}."
            put(P + "ln1", full.f32[P + "ln1"])
            put(P + "ln2", full.f32[P + "ln2"])
            put(P + "wqkv", src[P + "wqkv"].index_select(0, rows))
            if cfg.qkv_bias:
                put(P + "bqkv", full.f32[P + "bqkv"].index_select(0, rows))
            put(P + "wo", src[P + "wo"][:, q0:q0 + self.q_dim])
            put(P + "wgu", src[P + "wgu"][2 * f0:2 * (f0 + self.F)])
            put(P + "wdown", src[P + "wdown"][:, f0:f0 + self.F])
        if self.flat is None:
            self._make_views()

    def frozen_copy(self) -> "TPTrainLM":
        """A bf16-only copy of the current shard (the frozen reference policy)."""
        return TPTrainLM.__new__(TPTrainLM)._init_copy(self)

    def _init_copy(self, src: "TPTrainLM") -> "TPTrainLM":
        for k in ("cfg", "comm", "tp", "rank", "device", "layers", "hq", "hk", "q_dim", "kv_dim", "qkv_dim", "F",
                  "table", "offsets", "rep_numel", "numel", "has_embed", "has_head"):
            setattr(self, k, getattr(src, k))
        self.has_master = False
        self.flat, self.grad, self.shadow = None, None, src.shadow.clone()
        self._make_views()
        self.full = _Replicated(self)
        self._ws = {}
        return self

    def zero_grad(self):
        if self.grad is not None:
            self.grad.zero_()

    def sync_shadow(self):
        if self.flat is not None:
            self.shadow.copy_(self.flat)

    def head_weight(self):
        return self.full.head_weight()

    def head_grad(self):
        return self.full.head_grad()

    def reduce_replicated_grads(self):
        """Sums the partial gradients of the replicated parameters (embedding,
        norms, head: each rank saw only its rows) over the TP group."""
        import torch.distributed as dist

        if self.tp > 1:
            dist.all_reduce(self.grad[: self.rep_numel], group=self.comm.group)

    def _buf(self, key, shape, dtype=torch.bfloat16):
        t = self._ws.get(key)
        n = math.prod(shape)
        if t is None or t.numel() < n or t.dtype != dtype:
            t = torch.empty(n, device=self.device, dtype=dtype)
            self._ws[key] = t
        return t[:n].view(shape)

    # ------------------------------------------------------------------ training forward / backward
    def forward_train(self, x: torch.Tensor, B: int, T: int, pos_full: torch.Tensor, save: bool = True):
        """Forward of this rank's rows x [B*T/tp, H]; with save=True also returns
        what :meth:`backward` needs (one dict per layer)."""
        if not save:
            return self.forward(x, B, T, pos_full), None
        o, cfg, c = _ops(), self.cfg, self.comm
        N = B * T
        m = x.shape[0]
        H, D = cfg.hidden, cfg.head_dim
        scale = 1.0 / math.sqrt(D)
        bf = dict(device=self.device, dtype=torch.bfloat16)
        saved = []
        for i in self.layers:
            P = f"l{i}."
            w = self.w
            a = {"x": x, "h1": torch.empty(m, H, **bf), "r1": torch.empty(m, device=self.device),
                 "h1f": torch.empty(N, H, **bf), "qkv": torch.empty(N, self.qkv_dim, **bf),
                 "attn": torch.empty(N, self.q_dim, **bf), "lse": torch.empty(B * self.hq * T, device=self.device),
                 "h2": torch.empty(m, H, **bf), "r2": torch.empty(m, device=self.device),
                 "h2f": torch.empty(N, H, **bf), "gu": torch.empty(N, 2 * self.F, **bf),
                 "act": torch.empty(N, self.F, **bf)}
            o.rmsnorm_fwd(x, w[P + "ln1"], a["h1"], a["r1"], cfg.rms_eps)
            if cfg.qkv_bias:
                c.all_gather_gemm(a["h1"], w[P + "wqkv"], out=a["qkv"], bias=w[P + "bqkv"], epi=o.EPI_BIAS,
                                  gather_out=a["h1f"])
            else:
                c.all_gather_gemm(a["h1"], w[P + "wqkv"], out=a["qkv"], gather_out=a["h1f"])
            qkv = a["qkv"]
            o.rope(qkv, pos_full, self.table, self.hq + self.hk, D)
            q, k, v = qkv[:, : self.q_dim], qkv[:, self.q_dim:self.q_dim + self.kv_dim], qkv[:, self.q_dim + self.kv_dim:]
            o.flash_attn_fwd(q, k, v, a["attn"], a["lse"], B, T, self.hq, self.hk, scale)
            a["x2"] = c.gemm_reduce_scatter(a["attn"], w[P + "wo"], residual=x)
            o.rmsnorm_fwd(a["x2"], w[P + "ln2"], a["h2"], a["r2"], cfg.rms_eps)
            c.all_gather_gemm(a["h2"], w[P + "wgu"], out=a["act"], epi=o.EPI_SWIGLU, gather_out=a["h2f"],
                              c2=a["gu"])
            x = c.gemm_reduce_scatter(a["act"], w[P + "wdown"], residual=a["x2"])
            saved.append(a)
        return x, saved

    def backward(self, dx: torch.Tensor, saved, B: int, T: int, pos_full: torch.Tensor) -> torch.Tensor:
        """Backward through the layers; dx is d loss / d output for this rank's
        rows.  Accumulates this rank's weight gradients (replicated ones
        partially, see :meth:`reduce_replicated_grads`); returns d loss / d input rows."""
        o, cfg, c = _ops(), self.cfg, self.comm
        N = B * T
        m = dx.shape[0]
        H, D = cfg.hidden, cfg.head_dim
        scale = 1.0 / math.sqrt(D)
        G, w = self.g, self.w
        d_act = self._buf("d_act", (N, self.F))
        d_gu = self._buf("d_gu", (N, 2 * self.F))
        dfull = self._buf("dfull", (N, H))
        d_attn = self._buf("d_attn", (N, self.q_dim))
        d_qkv = self._buf("d_qkv", (N, self.qkv_dim))
        delta = self._buf("delta", (B * self.hq * T,), torch.float32)
        attn_ws = self._buf("attn_ws", (o.flash_attn_bwd_ws_numel(B, T, self.hk),), torch.float32)
        for i, a in zip(reversed(self.layers), reversed(saved)):
            P = f"l{i}."
            # ---- MLP: row-parallel down projection, column-parallel gate/up
            c.all_gather_gemm(dx, w[P + "wdown"], out=d_act, b_mn=True, gather_out=dfull)   # d act = dX Wdown_r
            o.gemm(dfull, a["act"], G[P + "wdown"], True, True, accumulate=True, split_k=1)  # dWdown_r += dX^T act
            o.swiglu_bwd(a["gu"], d_act, d_gu)
            dh2 = c.gemm_reduce_scatter(d_gu, w[P + "wgu"], b_mn=True)                     # dh2_r = RS(dGU Wgu_r)
            o.gemm(d_gu, a["h2f"], G[P + "wgu"], True, True, accumulate=True, split_k=1)   # dWgu_r += dGU^T h2
            dx2 = torch.empty(m, H, device=self.device, dtype=torch.bfloat16)
            o.rmsnorm_bwd(dh2, a["x2"], w[P + "ln2"], a["r2"], dx2, dx, G[P + "ln2"])
            # ---- attention: row-parallel output projection, column-parallel QKV
            c.all_gather_gemm(dx2, w[P + "wo"], out=d_attn, b_mn=True, gather_out=dfull)   # d attn = dX2 Wo_r
            o.gemm(dfull, a["attn"], G[P + "wo"], True, True, accumulate=True, split_k=1)  # dWo_r += dX2^T attn
            qkv = a["qkv"]
            q, k, v = qkv[:, : self.q_dim], qkv[:, self.q_dim:self.q_dim + self.kv_dim], qkv[:, self.q_dim + self.kv_dim:]
            dq = d_qkv[:, : self.q_dim]
            dk = d_qkv[:, self.q_dim:self.q_dim + self.kv_dim]
            dv = d_qkv[:, self.q_dim + self.kv_dim:]
            o.flash_attn_bwd(q, k, v, a["attn"], d_attn, a["lse"], delta, dq, dk, dv, B, T, self.hq, self.hk, scale,
                             ws=attn_ws)
            o.rope(d_qkv, pos_full, self.table, self.hq + self.hk, D, True)              # inverse rotation
            dh1 = c.gemm_reduce_scatter(d_qkv, w[P + "wqkv"], b_mn=True)                   # dh1_r = RS(dQKV Wqkv_r)
            o.gemm(d_qkv, a["h1f"], G[P + "wqkv"], True, True, accumulate=True, split_k=1)  # dWqkv_r += dQKV^T h1
            if cfg.qkv_bias:
                o.colsum_bf16(d_qkv, G[P + "bqkv"], True)
            dxi = torch.empty(m, H, device=self.device, dtype=torch.bfloat16)
            o.rmsnorm_bwd(dh1, a["x"], w[P + "ln1"], a["r1"], dxi, dx2, G[P + "ln1"])
            dx = dxi
        return dx

    def embed_backward_rows(self, ids_flat: torch.Tensor, dx: torch.Tensor):
        """Embedding gradient of this rank's rows (partial; summed over the group
        by :meth:`reduce_replicated_grads`)."""
        r0, m = self.rows_of(ids_flat.numel())
        _ops().embed_bwd(ids_flat[r0:r0 + m].to(torch.int32).contiguous(), dx, self.g["embed"])

    def state_dict(self):
        return {"cfg": self.cfg.__dict__, "layers": self.layers, "tp": self.tp, "rank": self.rank,
                "flat": self.flat, "shadow": self.shadow}

    def load_state_dict(self, sd):
        if self.flat is not None and sd.get("flat") is not None:
            self.flat.copy_(sd["flat"])
        self.shadow.copy_(sd["shadow"])
        if self.flat is None:
            self._make_views()
