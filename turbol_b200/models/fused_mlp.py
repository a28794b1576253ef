"""Tensor-core actor-critic MLP with hand-written forward and backward.

Two tanh MLPs (actor obs -> H -> H -> A logits, critic obs -> H -> H -> 1)
run on the tcgen05 GEMM (:func:`turbol_b200.ops.gemm`) with the pointwise work
fused into the GEMM epilogues:

  forward   H1 = tanh(X W1^T + b1)          one GEMM for actor and critic (W1 stacked)
            H2 = tanh(H1 W2^T + b2)         per head
            out = H2 W3^T + b3              per head (fp32)
  backward  dZ2 = (dOut W3) * (1 - H2^2)    GEMM + tanh-backward epilogue
            dZ1 = (dZ2 W2) * (1 - H1^2)     GEMM + tanh-backward epilogue
            dW  = dZ^T H                    MN-major x MN-major GEMM, split-K, fp32
            db  = column sums of dZ
No transposes are materialized and no [B, H] fp32 intermediates exist:
activations and activation gradients are bf16, weights are the bf16 shadow
that the fused Adam writes next to the fp32 master copy, and weight gradients
land in fp32 directly in the flat gradient buffer.

Shapes are padded for the tensor-core path: observations to 8 features and
the output heads to 8 rows (zero padding stays zero: its gradients are zero).
"""
from __future__ import annotations

import math
from typing import Sequence

import torch
import torch.nn as nn

from .._native import ops as _ops

PAD = 8


class FusedActorCritic:
    def __init__(self, obs_dim: int, act_dim: int, hidden: Sequence[int] = (256, 256), device="cuda",
                 seed: int = 0):
        if len(hidden) != 2 or hidden[0] != hidden[1]:
            raise ValueError("the fused MLP expects two equal hidden layers")
        H = int(hidden[0])
        if H % 64 or obs_dim > PAD or act_dim > PAD:
            raise ValueError("hidden must be a multiple of 64, obs_dim and act_dim at most 8")
        self.obs_dim, self.act_dim, self.H = obs_dim, act_dim, H
        self.device = torch.device(device)
        # parameter layout in the flat buffer; every offset 64-element aligned
        shapes = [("w1", (2 * H, PAD)), ("b1", (2 * H,)),
                  ("w2a", (H, H)), ("b2a", (H,)), ("w3a", (PAD, H)), ("b3a", (PAD,)),
                  ("w2c", (H, H)), ("b2c", (H,)), ("w3c", (PAD, H)), ("b3c", (PAD,))]
        self.offsets, off = {}, 0
        for name, shp in shapes:
            self.offsets[name] = (off, shp)
            off += (math.prod(shp) + 63) // 64 * 64
        self.numel = off
        self.flat = torch.zeros(off, device=self.device, dtype=torch.float32)
        self.grad = torch.zeros(off, device=self.device, dtype=torch.float32)
        self.shadow = torch.zeros(off, device=self.device, dtype=torch.bfloat16)
        self.p = {n: self._view(self.flat, n) for n in self.offsets}
        self.g = {n: self._view(self.grad, n) for n in self.offsets}
        self.s = {n: self._view(self.shadow, n) for n in self.offsets}
        self.reset_parameters(seed)
        self._ws = {}

    def rebind_storage(self, flat: torch.Tensor, grad: torch.Tensor, shadow: torch.Tensor):
        """Moves the weights into caller-owned buffers (e.g. NVLink peer memory)."""
        if flat.numel() < self.numel or grad.numel() < self.numel or shadow.numel() < self.numel:
            raise ValueError("rebind_storage: buffers too small")
        flat[: self.numel].copy_(self.flat)
        shadow[: self.numel].copy_(self.shadow)
        grad[: self.numel].zero_()
        self.flat, self.grad, self.shadow = flat[: self.numel], grad[: self.numel], shadow[: self.numel]
        self.p = {n: self._view(self.flat, n) for n in self.offsets}
        self.g = {n: self._view(self.grad, n) for n in self.offsets}
        self.s = {n: self._view(self.shadow, n) for n in self.offsets}

    def _view(self, buf, name):
        off, shp = self.offsets[name]
        return buf[off:off + math.prod(shp)].view(shp)

    # ------------------------------------------------------------ init / io
    def reset_parameters(self, seed: int = 0):
        gen = torch.Generator().manual_seed(seed)
        H, o, a = self.H, self.obs_dim, self.act_dim

        def orth(shape, gain):
            w = torch.empty(shape)
            nn.init.orthogonal_(w, gain=gain, generator=gen)
            return w

        with torch.no_grad():
            self.flat.zero_()
            # same draw order as ActorCritic: actor layers then critic layers
            w1a, w2a, w3a = orth((H, o), math.sqrt(2)), orth((H, H), math.sqrt(2)), orth((a, H), 0.01)
            w1c, w2c, w3c = orth((H, o), math.sqrt(2)), orth((H, H), math.sqrt(2)), orth((1, H), 1.0)
            self.p["w1"][:H, :o].copy_(w1a)
            self.p["w1"][H:, :o].copy_(w1c)
            self.p["w2a"].copy_(w2a)
            self.p["w3a"][:a].copy_(w3a)
            self.p["w2c"].copy_(w2c)
            self.p["w3c"][:1].copy_(w3c)
            self.sync_shadow()

    def sync_shadow(self):
        self.shadow.copy_(self.flat)

    def state_dict(self):
        return {"flat": self.flat.clone(), "offsets": {k: v for k, v in self.offsets.items()}}

    def load_state_dict(self, sd):
        self.flat.copy_(sd["flat"])
        self.sync_shadow()

    def to_actor_critic_params(self):
        """Unpadded (w, b) lists for actor and critic, for checks and export."""
        H, o, a = self.H, self.obs_dim, self.act_dim
        P = self.p
        actor = [P["w1"][:H, :o], P["b1"][:H], P["w2a"], P["b2a"], P["w3a"][:a], P["b3a"][:a]]
        critic = [P["w1"][H:, :o], P["b1"][H:], P["w2c"], P["b2c"], P["w3c"][:1], P["b3c"][:1]]
        return actor, critic

    # ------------------------------------------------------------ workspace
    def workspace(self, B: int):
        ws = self._ws.get(B)
        if ws is None:
            bf = dict(device=self.device, dtype=torch.bfloat16)
            f32 = dict(device=self.device, dtype=torch.float32)
            H = self.H
            ws = {
                "h1": torch.empty(B, 2 * H, **bf),
                "h2a": torch.empty(B, H, **bf),
                "h2c": torch.empty(B, H, **bf),
                "logits": torch.empty(B, PAD, **f32),
                "value": torch.empty(B, PAD, **f32),
                "dz2a": torch.empty(B, H, **bf),
                "dz2c": torch.empty(B, H, **bf),
                "dz1": torch.empty(B, 2 * H, **bf),
                "dlog": torch.empty(B, PAD, **bf),
                "dval": torch.empty(B, PAD, **bf),
            }
            o = _ops()
            n = max(o.gemm_workspace_numel(H, H, B), o.gemm_workspace_numel(PAD, H, B),
                    o.gemm_workspace_numel(2 * H, PAD, B), 1)
            # split-K partials of the weight-gradient GEMMs (zero-filled: its
            # head holds arrival counters that every call leaves zero)
            ws["splitk"] = torch.zeros(n, **f32)
            self._ws[B] = ws
        return ws

    # ------------------------------------------------------------ compute
    def forward(self, x_bf16: torch.Tensor, ws=None):
        """x_bf16 [B, 8] -> (logits fp32 [B, 8], value fp32 [B, 8] (column 0))."""
        o = _ops()
        B = x_bf16.shape[0]
        ws = ws or self.workspace(B)
        S, P = self.s, self.p
        H = self.H
        h1 = ws["h1"]
        o.dense_k8_fwd(x_bf16, S["w1"], P["b1"], h1, True)                 # 8 input features: CUDA cores
        o.gemm(h1[:, :H], S["w2a"], ws["h2a"], bias=P["b2a"], epi=o.EPI_BIAS_TANH)
        o.gemm(h1[:, H:], S["w2c"], ws["h2c"], bias=P["b2c"], epi=o.EPI_BIAS_TANH)
        o.gemm(ws["h2a"], S["w3a"], ws["logits"], bias=P["b3a"], epi=o.EPI_BIAS)
        o.gemm(ws["h2c"], S["w3c"], ws["value"], bias=P["b3c"], epi=o.EPI_BIAS)
        return ws["logits"], ws["value"]

    def backward(self, x_bf16: torch.Tensor, ws, out_bias_grads_done: bool = False):
        """Weight gradients into self.grad from ws['dlog'] / ws['dval'] (bf16 [B, 8]).

        The hidden-layer bias gradients come out of the tanh-backward GEMM
        epilogues (column sums); the output-layer bias gradients come from the
        loss kernel when ``out_bias_grads_done`` (else a column-sum kernel)."""
        o = _ops()
        S, G = self.s, self.g
        H = self.H
        h1, wsk = ws["h1"], ws["splitk"]
        for head, dout, h2, dz2, w2, w3, cols in (("a", ws["dlog"], ws["h2a"], ws["dz2a"], S["w2a"], S["w3a"], slice(0, H)),
                                                   ("c", ws["dval"], ws["h2c"], ws["dz2c"], S["w2c"], S["w3c"], slice(H, 2 * H))):
            o.gemm(dout, h2, G["w3" + head], True, True, workspace=wsk)          # dW3 = dOut^T H2
            if not out_bias_grads_done:
                o.colsum_bf16(dout, G["b3" + head])                                # db3
            o.gemm(dout, w3, dz2, False, True, aux=h2, epi=o.EPI_TANH_BWD,        # dZ2 = (dOut W3)(1 - H2^2)
                   colsum=G["b2" + head])                                          #   db2 = sum dZ2
            o.gemm(dz2, h1[:, cols], G["w2" + head], True, True, workspace=wsk)   # dW2 = dZ2^T H1
            o.gemm(dz2, w2, ws["dz1"][:, cols], False, True, aux=h1[:, cols],     # dZ1 = (dZ2 W2)(1 - H1^2)
                   epi=o.EPI_TANH_BWD, colsum=G["b1"][cols])                       #   db1 = sum dZ1
        o.gemm(ws["dz1"], x_bf16, G["w1"], True, True, workspace=wsk)             # dW1 = dZ1^T X
