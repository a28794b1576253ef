"""Tensor-core actor-critic MLP with hand-written forward and backward.

Two tanh MLPs (actor obs -> H -> H -> A logits, critic obs -> H -> H -> 1)
run as one network with block-diagonal layers: the actor and the critic are
the two diagonal blocks of W2 and W3 [16, 2H], so every layer is a single
launch for both heads.  W2 stores only its two [H, H] diagonal blocks, packed
as [2H, H] (the GEMM's packed `kgroup` operand), so neither the optimizer nor
the data-parallel exchange touches the zero off-diagonal half; W3's
off-diagonal blocks are zero and receive no gradient, so they stay zero.  The 8-feature first layer runs on CUDA cores
(a tensor-core tile would be mostly K padding); the rest on the tcgen05 GEMM
(:func:`turbol_b200.ops.gemm`) with the pointwise work fused into the GEMM
epilogues:

  forward   H1 = tanh(X W1^T + b1)          [B, 2H], CUDA-core kernel
            H2 = tanh(H1 W2^T + b2)         [B, 2H], one GEMM over the diagonal
                                            blocks only (kgroup: each output tile
                                            iterates over its head's K range and
                                            reads its head's packed block)
            out = H2 W3^T + b3              [B, 16] fp32 (logits | value), one GEMM
  training  with 2 actions and H in {128, 256}: output layer + clipped PPO loss +
            dZ2, dW3, db3, db2 in ONE CUDA-core pass over H2 (ppo_head.cu:
            :meth:`forward_hidden` + :meth:`loss_backward`), then dW2, dZ1, dW1
  backward  dZ2 = (dOut W3) * (1 - H2^2)    one CUDA-core pass (8 outputs per head) + db2 column sums
            dW3 = dOut^T H2                 one CUDA-core pass (8 rows per head, 18.6 vs 36.8 us as GEMMs)
            dZ1 = (dZ2 W2) * (1 - H1^2)     one GEMM (diagonal blocks only) + tanh-backward
                                            epilogue (+ db1 column sums)
            dW2, dW1 = dZ^T H               MN-major x MN-major GEMMs, split-K, fp32
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
        # the one-pass output layer + loss + output-layer backward (ppo_head.cu)
        self.fused_head = act_dim == 2 and H in (128, 256)
        # parameter layout in the flat buffer; every offset 64-element aligned
        # W2 holds only the two diagonal blocks, packed: rows [0, H) are the
        # actor's [H, H] block, rows [H, 2H) the critic's
        shapes = [("w1", (2 * H, PAD)), ("b1", (2 * H,)), ("w2", (2 * H, H)), ("b2", (2 * H,)),
                  ("w3", (2 * PAD, 2 * H)), ("b3", (2 * PAD,))]
        self.offsets, off = {}, 0
        for name, shp in shapes:
            self.offsets[name] = (off, shp)
            off += (math.prod(shp) + 63) // 64 * 64
        self.numel = off
        self.flat = torch.zeros(off, device=self.device, dtype=torch.float32)
        self.grad = torch.zeros(off, device=self.device, dtype=torch.float32)
        self.shadow = torch.zeros(off, device=self.device, dtype=torch.bfloat16)
        self._make_views()
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
        self._make_views()

    def _view(self, buf, name):
        off, shp = self.offsets[name]
        return buf[off:off + math.prod(shp)].view(shp)

    def _make_views(self):
        """Whole parameters plus per-head views of the diagonal blocks
        (w2a / w2c, b2a / b2c, w3a / w3c, b3a / b3c)."""
        H = self.H

        def views(buf):
            d = {n: self._view(buf, n) for n in self.offsets}
            d["w2a"], d["w2c"] = d["w2"][:H], d["w2"][H:]
            d["b2a"], d["b2c"] = d["b2"][:H], d["b2"][H:]
            d["w3a"], d["w3c"] = d["w3"][:PAD, :H], d["w3"][PAD:, H:]
            d["b3a"], d["b3c"] = d["b3"][:PAD], d["b3"][PAD:]
            return d

        self.p, self.g, self.s = views(self.flat), views(self.grad), views(self.shadow)

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
            out = torch.empty(B, 2 * PAD, **f32)       # logits | value
            dout = torch.empty(B, 2 * PAD, **bf)       # d logits | d value
            ws = {
                "h1": torch.empty(B, 2 * H, **bf),
                "h2": torch.empty(B, 2 * H, **bf),
                "out": out, "logits": out[:, :PAD], "value": out[:, PAD:],
                "dz2": torch.empty(B, 2 * H, **bf),
                "dz1": torch.empty(B, 2 * H, **bf),
                "dout": dout, "dlog": dout[:, :PAD], "dval": dout[:, PAD:],
            }
            o = _ops()
            n = max(o.gemm_workspace_numel(H, H, B), o.gemm_workspace_numel(PAD, H, B),
                    o.gemm_workspace_numel(2 * H, PAD, B), 1)
            # split-K partials of the weight-gradient GEMMs (zero-filled: its
            # head holds arrival counters that every call leaves zero)
            ws["splitk"] = torch.zeros(n, **f32)
            # per-CTA partial sums of the 8-wide CUDA-core passes
            ws["parts"] = torch.empty(o.skinny8_scratch_numel(min(2 * H, 512)), **f32)
            if self.fused_head:
                ws["head_parts"] = o.ppo_head_parts(H, self.act_dim)
                ws["head_part"] = torch.empty(o.ppo_head_part_numel(H, self.act_dim, ws["head_parts"]), **f32)
            self._ws[B] = ws
        return ws

    # ------------------------------------------------------------ compute
    def forward(self, x_bf16: torch.Tensor, ws=None):
        """x_bf16 [B, 8] -> (logits fp32 [B, 8], value fp32 [B, 8] (column 0)), views of ws['out']."""
        o = _ops()
        B = x_bf16.shape[0]
        ws = ws or self.workspace(B)
        S, P = self.s, self.p
        o.dense_k8_fwd(x_bf16, S["w1"], P["b1"], ws["h1"], True)                 # 8 input features: CUDA cores
        # both heads' hidden layer (128-wide tiles: 34.2 vs 37.3 us at 32,768 rows); kgroup=H: each
        # output tile reads only its head's diagonal block of W2 (half the MMAs and operand loads)
        o.gemm(ws["h1"], S["w2"], ws["h2"], bias=P["b2"], epi=o.EPI_BIAS_TANH, bn=128, kgroup=self.H)
        # (the CUDA-core mlp_head_fwd measured slower here: 26.7 vs 16.5 us at 32,768 rows)
        o.gemm(ws["h2"], S["w3"], ws["out"], bias=P["b3"], epi=o.EPI_BIAS)        # logits | value
        return ws["logits"], ws["value"]

    def forward_hidden(self, x_bf16: torch.Tensor, ws):
        """The two hidden layers only: ws['h1'], ws['h2'] (the input of :meth:`loss_backward`)."""
        o = _ops()
        S, P = self.s, self.p
        o.dense_k8_fwd(x_bf16, S["w1"], P["b1"], ws["h1"], True)
        o.gemm(ws["h1"], S["w2"], ws["h2"], bias=P["b2"], epi=o.EPI_BIAS_TANH, bn=128, kgroup=self.H)

    def loss_backward(self, x_bf16: torch.Tensor, ws, act, old_logp, adv, ret, stats, clip: float, vf_coef: float,
                      ent_coef: float):
        """Output layer, clipped PPO loss and the whole backward after
        :meth:`forward_hidden`: one pass over H2 computes the logits and values,
        the loss (statistics added into ``stats``), dZ2 and the gradients of W3,
        b3 and b2 (ppo_head.cu); then the GEMMs for dW2, dZ1 (+ db1) and dW1."""
        o = _ops()
        S, G, P = self.s, self.g, self.p
        o.ppo_head(ws["h2"], S["w3"], P["b3"], PAD, self.act_dim, act, old_logp, adv, ret, ws["dz2"], G["w3"], G["b3"],
                   G["b2"], stats, ws["head_part"], ws["head_parts"], clip, vf_coef, ent_coef)
        self._hidden_backward(x_bf16, ws)

    def _hidden_backward(self, x_bf16: torch.Tensor, ws):
        """dW2 (per head), dZ1 + db1 and dW1 from ws['dz2']."""
        o = _ops()
        S, G = self.s, self.g
        H = self.H
        h1, dz2, dz1, wsk = ws["h1"], ws["dz2"], ws["dz1"], ws["splitk"]
        # dW2 block = dZ2^T H1 (128-wide tiles, 32 K splits: 35.1 vs 42.9 us for both heads at 32,768 rows)
        for head, cols in (("a", slice(0, H)), ("c", slice(H, 2 * H))):
            o.gemm(dz2[:, cols], h1[:, cols], G["w2" + head], True, True, workspace=wsk, bn=128, split_k=32)
        o.gemm(dz2, S["w2"], dz1, False, True, aux=h1, epi=o.EPI_TANH_BWD, colsum=G["b1"],   # dZ1, db1
               kgroup=self.H)                                                    # (packed diagonal blocks of W2)
        o.gemm(dz1, x_bf16, G["w1"], True, True, workspace=wsk)                              # dW1 = dZ1^T X

    def backward(self, x_bf16: torch.Tensor, ws, out_bias_grads_done: bool = False):
        """Weight gradients into self.grad from ws['dout'] = (d logits | d value)
        (bf16 [B, 16]).

        The hidden-layer bias gradients come out of the tanh-backward GEMM
        epilogues (column sums); the output-layer bias gradients come from the
        loss kernel when ``out_bias_grads_done`` (else a column-sum kernel).
        W3's gradient is computed for its diagonal blocks only, so its
        off-diagonal gradient (and weights) stay zero."""
        o = _ops()
        S, G = self.s, self.g
        H = self.H
        h1, h2, dz2, dz1, dout, wsk = ws["h1"], ws["h2"], ws["dz2"], ws["dz1"], ws["dout"], ws["splitk"]
        narrow = 2 * H <= 512  # the CUDA-core passes keep a whole row of H2 in one CTA's column threads
        if narrow:
            # dW3 diagonal blocks = dOut_head^T H2_head (8 rows per head): one CUDA-core
            # pass over H2 (a tensor-core tile would be 15/16 padding)
            o.skinny8_wgrad(h2, dout, G["w3"], H, 1, 2 * H, PAD * 2 * H, False, ws["parts"])
        else:
            for head, rows, cols in (("a", slice(0, PAD), slice(0, H)), ("c", slice(PAD, 2 * PAD), slice(H, 2 * H))):
                o.gemm(dout[:, rows], h2[:, cols], G["w3" + head], True, True, workspace=wsk)  # dW3 = dOut^T H2
        if not out_bias_grads_done:
            o.colsum_bf16(dout, G["b3"])
        if narrow:  # dZ2 = (dOut W3) * (1 - H2^2), db2: K = 8 per head, one CUDA-core pass
            o.mlp_head_dz(dout, h2, S["w3"], H, dz2, G["b2"], False, ws["parts"])
        else:
            o.gemm(dout, S["w3"], dz2, False, True, aux=h2, epi=o.EPI_TANH_BWD, colsum=G["b2"])
        self._hidden_backward(x_bf16, ws)
