"""Decoder-only transformer (Qwen2 / Llama family) on the turbol_b200 kernels.

Architecture: token embedding -> L x [RMSNorm -> fused QKV projection (+bias)
-> RoPE -> causal GQA attention -> output projection (+residual) -> RMSNorm ->
gate/up projection -> SwiGLU -> down projection (+residual)] -> RMSNorm ->
LM head (tied to the embedding or separate).

Weights live in one flat fp32 master buffer with a bf16 copy (what the
GEMMs read) and a flat fp32 gradient buffer, so the optimizer, data-parallel
reduction, checkpointing and trainer->rollout weight sync each touch one
contiguous buffer.  The gate and up projections are stored interleaved row by
row (gate_j, up_j), which lets the decode path fuse SwiGLU into the GEMM
epilogue.

Forward and backward are written by hand (no autograd): every projection is a
tcgen05 GEMM with its pointwise work fused into the epilogue (bias, residual
add), weight gradients accumulate in fp32 straight into the gradient buffer,
and activations are bf16.  A model instance can hold a slice of the layers
(pipeline stages) and optionally the embedding / head.

Reference parity: the reference has no LLM training path (its PolicyEngine is
a linear policy, turbol_vllm/src/policy/policy_engine.cpp); this module is the
policy the GRPO / PPO-RLHF configurations need.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional, Sequence

import torch

from .._native import ops as _ops

ALIGN = 64  # elements; every parameter offset is 128-byte aligned in bf16


@dataclass
class LMConfig:
    n_layers: int = 28
    hidden: int = 1536
    n_heads: int = 12
    n_kv_heads: int = 2
    head_dim: int = 128
    ffn: int = 8960
    vocab: int = 151936
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    tie_embeddings: bool = True
    qkv_bias: bool = True
    max_seq: int = 4096
    init_std: float = 0.02

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    @staticmethod
    def qwen2_1p5b() -> "LMConfig":
        """28 layers, hidden 1536, 12 q / 2 kv heads, SwiGLU 8960, vocab 151,936, RoPE 1e6."""
        return LMConfig()

    @staticmethod
    def llama3_8b() -> "LMConfig":
        """32 layers, hidden 4096, 32 q / 8 kv heads, SwiGLU 14,336, vocab 128,256, RoPE 5e5."""
        return LMConfig(n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8, ffn=14336, vocab=128256,
                        rope_theta=5e5, rms_eps=1e-5, tie_embeddings=False, qkv_bias=False)

    @staticmethod
    def tiny(n_layers: int = 2, vocab: int = 1024) -> "LMConfig":
        return LMConfig(n_layers=n_layers, hidden=256, n_heads=4, n_kv_heads=2, ffn=512, vocab=vocab,
                        rope_theta=1e4, max_seq=1024)

    def param_count(self) -> int:
        H, L = self.hidden, self.n_layers
        per = 2 * H + self.qkv_dim * H + (self.qkv_dim if self.qkv_bias else 0) + H * self.q_dim + 3 * self.ffn * H
        return L * per + self.vocab * H * (1 if self.tie_embeddings else 2) + H


def rope_table(cfg: LMConfig, device) -> torch.Tensor:
    """[max_seq, head_dim/2, 2] fp32 (cos, sin) for rotate-half RoPE."""
    D = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = torch.arange(cfg.max_seq, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.stack([torch.cos(ang), torch.sin(ang)], -1).to(device=device, dtype=torch.float32).contiguous()


class DecoderLM:
    def __init__(self, cfg: LMConfig, device="cuda", layers: Optional[Sequence[int]] = None, embed: bool = True,
                 head: bool = True, seed: int = 0, master: bool = True, storage: Optional[Dict] = None):
        """layers: indices of the layers this instance holds (default all);
        master=False keeps only the bf16 weights (a frozen reference copy)."""
        self.cfg = cfg
        self.device = torch.device(device)
        self.layers = list(range(cfg.n_layers)) if layers is None else list(layers)
        self.has_embed, self.has_head = embed, head
        self.has_master = master
        self.offsets: Dict[str, tuple] = {}
        off = 0

        def add(name, shape):
            nonlocal off
            self.offsets[name] = (off, tuple(shape))
            off += (math.prod(shape) + ALIGN - 1) // ALIGN * ALIGN

        H, F = cfg.hidden, cfg.ffn
        if embed or (head and cfg.tie_embeddings):
            add("embed", (cfg.vocab, H))
        for i in self.layers:
            add(f"l{i}.ln1", (H,))
            add(f"l{i}.wqkv", (cfg.qkv_dim, H))
            if cfg.qkv_bias:
                add(f"l{i}.bqkv", (cfg.qkv_dim,))
            add(f"l{i}.wo", (H, cfg.q_dim))
            add(f"l{i}.ln2", (H,))
            add(f"l{i}.wgu", (2 * F, H))
            add(f"l{i}.wdown", (H, F))
        if head:
            add("norm", (H,))
            if not cfg.tie_embeddings:
                add("lm_head", (cfg.vocab, H))
        self.numel = off
        if storage is not None:
            self.flat, self.grad, self.shadow = storage["flat"], storage["grad"], storage["shadow"]
        else:
            self.shadow = torch.zeros(off, device=self.device, dtype=torch.bfloat16)
            self.flat = torch.zeros(off, device=self.device, dtype=torch.float32) if master else None
            self.grad = torch.zeros(off, device=self.device, dtype=torch.float32) if master else None
        self._make_views()
        self.table = rope_table(cfg, self.device)
        if storage is None:
            self.reset_parameters(seed)
        self._ws: Dict = {}

    # ------------------------------------------------------------------ params
    def _make_views(self):
        def views(buf):
            if buf is None:
                return None
            return {n: buf[o:o + math.prod(s)].view(s) for n, (o, s) in self.offsets.items()}

        self.p, self.g, self.s = views(self.flat), views(self.grad), views(self.shadow)
        # fp32 norm weights and biases are read by the kernels; a frozen copy
        # without master weights keeps fp32 versions of just those
        if self.flat is None:
            self.f32 = {n: self.s[n].float() for n in self.offsets if n.endswith(("ln1", "ln2", "norm", "bqkv"))}
        else:
            self.f32 = self.p

    def rebind_storage(self, flat, grad, shadow):
        if flat is not None:
            flat[: self.numel].copy_(self.flat)
        shadow[: self.numel].copy_(self.shadow)
        if grad is not None:
            grad[: self.numel].zero_()
        self.flat = flat[: self.numel] if flat is not None else None
        self.grad = grad[: self.numel] if grad is not None else None
        self.shadow = shadow[: self.numel]
        self._make_views()

    def reset_parameters(self, seed: int = 0):
        gen = torch.Generator(device=self.device).manual_seed(seed)
        std = self.cfg.init_std
        with torch.no_grad():
            for name, (off, shape) in self.offsets.items():
                tgt = self.p[name] if self.flat is not None else None
                if name.endswith(("ln1", "ln2", "norm")):
                    val = torch.ones(shape, device=self.device)
                elif name.endswith("bqkv"):
                    val = torch.zeros(shape, device=self.device)
                else:
                    val = torch.randn(shape, device=self.device, generator=gen) * std
                    if name.endswith(("wo", "wdown")):
                        val *= 1.0 / math.sqrt(2 * self.cfg.n_layers)
                if tgt is not None:
                    tgt.copy_(val)
                self.s[name].copy_(val)
        if self.flat is None:
            self._make_views()

    def sync_shadow(self):
        if self.flat is not None:
            self.shadow.copy_(self.flat)

    def frozen_copy(self) -> "DecoderLM":
        """A bf16-only copy of the current weights (the GRPO reference model)."""
        ref = DecoderLM(self.cfg, self.device, self.layers, self.has_embed, self.has_head, master=False,
                        storage={"flat": None, "grad": None, "shadow": self.shadow.clone()})
        return ref

    def head_weight(self):
        return self.s["embed"] if self.cfg.tie_embeddings else self.s["lm_head"]

    def head_grad(self):
        return self.g["embed"] if self.cfg.tie_embeddings else self.g["lm_head"]

    # ------------------------------------------------------------------ workspace
    def _buf(self, key, shape, dtype=torch.bfloat16):
        t = self._ws.get(key)
        n = math.prod(shape)
        if t is None or t.numel() < n or t.dtype != dtype:
            t = torch.empty(n, device=self.device, dtype=dtype)
            self._ws[key] = t
        return t[:n].view(shape)

    # ------------------------------------------------------------------ forward
    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        N = ids.numel()
        x = torch.empty(N, self.cfg.hidden, device=self.device, dtype=torch.bfloat16)
        _ops().embed_fwd(ids.reshape(-1).to(torch.int32).contiguous(), self.s["embed"], x)
        return x

    def forward(self, x: torch.Tensor, B: int, T: int, pos: torch.Tensor, save: bool = False, kv_hook=None):
        """Runs this instance's layers on the residual stream x [B*T, H] (bf16).
        Returns (x_out, saved) where saved holds what backward needs.
        kv_hook(layer, qkv) sees each layer's rotated QKV rows (prefill writes
        them into the paged KV cache)."""
        o = _ops()
        cfg = self.cfg
        N = B * T
        H, F, D = cfg.hidden, cfg.ffn, cfg.head_dim
        scale = 1.0 / math.sqrt(D)
        saved: List[Dict] = []
        for i in self.layers:
            P = f"l{i}."
            if save:
                a = {"x": x,
                     "h1": torch.empty(N, H, device=self.device, dtype=torch.bfloat16),
                     "r1": torch.empty(N, device=self.device),
                     "qkv": torch.empty(N, cfg.qkv_dim, device=self.device, dtype=torch.bfloat16),
                     "attn": torch.empty(N, cfg.q_dim, device=self.device, dtype=torch.bfloat16),
                     "lse": torch.empty(B * cfg.n_heads * T, device=self.device),
                     "x2": torch.empty(N, H, device=self.device, dtype=torch.bfloat16),
                     "h2": torch.empty(N, H, device=self.device, dtype=torch.bfloat16),
                     "r2": torch.empty(N, device=self.device),
                     "gu": torch.empty(N, 2 * F, device=self.device, dtype=torch.bfloat16),
                     "act": torch.empty(N, F, device=self.device, dtype=torch.bfloat16)}
            else:
                a = {"x": x, "h1": self._buf("h1", (N, H)), "r1": None, "qkv": self._buf("qkv", (N, cfg.qkv_dim)),
                     "attn": self._buf("attn", (N, cfg.q_dim)), "lse": None,
                     "x2": self._buf("x2", (N, H)), "h2": self._buf("h2", (N, H)), "r2": None,
                     "gu": None, "act": self._buf("act", (N, F))}
            o.rmsnorm_fwd(x, self.f32[P + "ln1"], a["h1"], a["r1"], cfg.rms_eps)
            qkv = a["qkv"]
            if cfg.qkv_bias:
                o.gemm(a["h1"], self.s[P + "wqkv"], qkv, bias=self.f32[P + "bqkv"], epi=o.EPI_BIAS)
            else:
                o.gemm(a["h1"], self.s[P + "wqkv"], qkv)
            o.rope(qkv, pos, self.table, cfg.n_heads + cfg.n_kv_heads, D)
            if kv_hook is not None:
                kv_hook(i, qkv)
            q, k, v = qkv[:, : cfg.q_dim], qkv[:, cfg.q_dim:cfg.q_dim + cfg.kv_dim], qkv[:, cfg.q_dim + cfg.kv_dim:]
            o.flash_attn_fwd(q, k, v, a["attn"], a["lse"], B, T, cfg.n_heads, cfg.n_kv_heads, scale)
            o.gemm(a["attn"], self.s[P + "wo"], a["x2"], aux=x, epi=o.EPI_RESIDUAL)
            o.rmsnorm_fwd(a["x2"], self.f32[P + "ln2"], a["h2"], a["r2"], cfg.rms_eps)
            if save:  # SwiGLU in the epilogue; the raw gate/up product is kept for the backward
                o.gemm(a["h2"], self.s[P + "wgu"], a["act"], epi=o.EPI_SWIGLU, c2=a["gu"])
            else:
                o.gemm(a["h2"], self.s[P + "wgu"], a["act"], epi=o.EPI_SWIGLU)
            xo = torch.empty(N, H, device=self.device, dtype=torch.bfloat16) if save else \
                self._buf("xo%d" % (len(saved) % 2), (N, H))
            o.gemm(a["act"], self.s[P + "wdown"], xo, aux=a["x2"], epi=o.EPI_RESIDUAL)
            if save:
                saved.append(a)
            else:
                saved.append(None)
            x = xo
        return x, saved

    def final_norm(self, x: torch.Tensor, rstd: Optional[torch.Tensor] = None) -> torch.Tensor:
        y = torch.empty_like(x)
        _ops().rmsnorm_fwd(x, self.f32["norm"], y, rstd, self.cfg.rms_eps)
        return y

    def logits(self, h: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """h [R, H] -> logits [R, V] bf16 (the caller chunks R)."""
        R = h.shape[0]
        if out is None:
            out = torch.empty(R, self.cfg.vocab, device=self.device, dtype=torch.bfloat16)
        _ops().gemm(h, self.head_weight(), out)
        return out

    # ------------------------------------------------------------------ backward
    def backward(self, dx: torch.Tensor, saved: List[Dict], B: int, T: int, pos: torch.Tensor) -> torch.Tensor:
        """Backward through this instance's layers; dx is d loss / d output
        (bf16 [B*T, H]).  Accumulates weight gradients; returns d loss / d input."""
        o = _ops()
        cfg = self.cfg
        N = B * T
        H, F, D = cfg.hidden, cfg.ffn, cfg.head_dim
        scale = 1.0 / math.sqrt(D)
        G = self.g
        d_gu = self._buf("d_gu", (N, 2 * F))
        dh = self._buf("dh", (N, H))
        d_attn = self._buf("d_attn", (N, cfg.q_dim))
        d_qkv = self._buf("d_qkv", (N, cfg.qkv_dim))
        delta = self._buf("delta", (B * cfg.n_heads * T,), torch.float32)
        attn_ws = self._buf("attn_ws", (o.flash_attn_bwd_ws_numel(B, T, cfg.n_kv_heads),), torch.float32)
        for i, a in zip(reversed(self.layers), reversed(saved)):
            P = f"l{i}."
            # ---- MLP
            # d act = dX Wdown, turned into d(gate, up) by the SwiGLU-backward epilogue
            o.gemm(dx, self.s[P + "wdown"], d_gu, False, True, aux=a["gu"], epi=o.EPI_SWIGLU_BWD)
            o.gemm(dx, a["act"], G[P + "wdown"], True, True, accumulate=True, split_k=1)  # dWdown += dX^T act
            o.gemm(d_gu, self.s[P + "wgu"], dh, False, True)                        # dh2 = dGU Wgu
            o.gemm(d_gu, a["h2"], G[P + "wgu"], True, True, accumulate=True, split_k=1)  # dWgu += dGU^T h2
            dx2 = torch.empty(N, H, device=self.device, dtype=torch.bfloat16)
            o.rmsnorm_bwd(dh, a["x2"], self.f32[P + "ln2"], a["r2"], dx2, dx, G[P + "ln2"])
            # ---- attention
            o.gemm(dx2, self.s[P + "wo"], d_attn, False, True)                      # d attn = dX2 Wo
            o.gemm(dx2, a["attn"], G[P + "wo"], True, True, accumulate=True, split_k=1)  # dWo += dX2^T attn
            qkv = a["qkv"]
            q, k, v = qkv[:, : cfg.q_dim], qkv[:, cfg.q_dim:cfg.q_dim + cfg.kv_dim], qkv[:, cfg.q_dim + cfg.kv_dim:]
            dq = d_qkv[:, : cfg.q_dim]
            dk = d_qkv[:, cfg.q_dim:cfg.q_dim + cfg.kv_dim]
            dv = d_qkv[:, cfg.q_dim + cfg.kv_dim:]
            o.flash_attn_bwd(q, k, v, a["attn"], d_attn, a["lse"], delta, dq, dk, dv, B, T, cfg.n_heads,
                             cfg.n_kv_heads, scale, ws=attn_ws)
            o.rope(d_qkv, pos, self.table, cfg.n_heads + cfg.n_kv_heads, D, True)   # inverse rotation
            o.gemm(d_qkv, self.s[P + "wqkv"], dh, False, True)                      # dh1 = dQKV Wqkv
            o.gemm(d_qkv, a["h1"], G[P + "wqkv"], True, True, accumulate=True, split_k=1)  # dWqkv += dQKV^T h1
            if cfg.qkv_bias:
                o.colsum_bf16(d_qkv, G[P + "bqkv"], True)
            dxi = torch.empty(N, H, device=self.device, dtype=torch.bfloat16)
            o.rmsnorm_bwd(dh, a["x"], self.f32[P + "ln1"], a["r1"], dxi, dx2, G[P + "ln1"])
            dx = dxi
        return dx

    def embed_backward(self, ids: torch.Tensor, dx: torch.Tensor):
        _ops().embed_bwd(ids.reshape(-1).to(torch.int32).contiguous(), dx, self.g["embed"])

    # ------------------------------------------------------------------ utilities
    def zero_grad(self):
        if self.grad is not None:
            self.grad.zero_()

    def state_dict(self):
        return {"cfg": self.cfg.__dict__, "layers": self.layers, "flat": self.flat if self.flat is not None else None,
                "shadow": self.shadow}

    def load_state_dict(self, sd):
        if self.flat is not None and sd.get("flat") is not None:
            self.flat.copy_(sd["flat"])
        self.shadow.copy_(sd["shadow"])
        if self.flat is None:
            self._make_views()
