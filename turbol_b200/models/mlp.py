"""MLP actor-critic networks with all parameters in one flat fp32 buffer.

One flat buffer (and one flat gradient buffer whose views are the parameters'
``.grad``) lets the optimizer and the data-parallel reduction treat the whole
model as a single contiguous bucket: one fused Adam launch, one peer-memory
all-reduce, no per-tensor bookkeeping.

The networks follow the usual PPO conventions: tanh hidden layers, orthogonal
initialization (gain sqrt(2) on hidden layers, 0.01 on the policy head, 1.0 on
the value head, zero biases), seeded from a ``torch.Generator`` so two runs
with the same seed start from identical weights.  The reference's
``PolicyEngine`` (turbol_vllm/src/policy/policy_engine.cpp:23-45) uses one
linear layer for each head; ``hidden=()`` reproduces that shape.
"""
from __future__ import annotations

import math
from typing import Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F


class FlatParameters:
    """Allocates parameters of the given shapes as views of one flat buffer."""

    def __init__(self, shapes: Sequence[Sequence[int]], device, dtype=torch.float32):
        self.shapes = [tuple(s) for s in shapes]
        self.numels = [math.prod(s) for s in self.shapes]
        total = sum(self.numels)
        # 16-byte aligned length so float4 kernels cover the buffer exactly
        self.numel = (total + 3) // 4 * 4
        self.flat = torch.zeros(self.numel, device=device, dtype=dtype)
        self.grad = torch.zeros(self.numel, device=device, dtype=dtype)
        self.params: list[nn.Parameter] = []
        off = 0
        for s, n in zip(self.shapes, self.numels):
            p = nn.Parameter(self.flat[off:off + n].view(s))
            p.grad = self.grad[off:off + n].view(s)
            self.params.append(p)
            off += n

    def zero_grad(self):
        self.grad.zero_()

    def rebind_grads(self):
        """Re-points every ``.grad`` at its view of the flat gradient buffer."""
        off = 0
        for p, n, s in zip(self.params, self.numels, self.shapes):
            p.grad = self.grad[off:off + n].view(s)
            off += n


def _orthogonal(shape, gain, gen):
    w = torch.empty(shape, dtype=torch.float32)
    nn.init.orthogonal_(w, gain=gain, generator=gen)
    return w


class ActorCritic(nn.Module):
    """Separate actor and critic MLPs: obs -> hidden... -> {act_dim logits | 1}.

    ``discrete=True`` gives a categorical policy over ``act_dim`` actions;
    ``discrete=False`` gives a Gaussian policy with mean ``tanh(actor(obs))``
    and a fixed std (the reference's continuous mode).
    """

    def __init__(self, obs_dim: int, act_dim: int, hidden: Sequence[int] = (64, 64), discrete: bool = True,
                 device="cpu", seed: int = 0, gaussian_std: float = 0.5):
        super().__init__()
        self.obs_dim, self.act_dim, self.hidden = obs_dim, act_dim, tuple(hidden)
        self.discrete, self.gaussian_std = discrete, gaussian_std
        dims_a = [obs_dim, *self.hidden, act_dim]
        dims_c = [obs_dim, *self.hidden, 1]
        shapes = []
        for dims in (dims_a, dims_c):
            for i in range(len(dims) - 1):
                shapes += [(dims[i + 1], dims[i]), (dims[i + 1],)]
        self.fp = FlatParameters(shapes, device)
        n_layers = len(dims_a) - 1
        self.actor_params = self.fp.params[: 2 * n_layers]
        self.critic_params = self.fp.params[2 * n_layers:]
        for i, p in enumerate(self.fp.params):
            self.register_parameter(f"p{i}", p)
        self.reset_parameters(seed)

    def reset_parameters(self, seed: int = 0):
        gen = torch.Generator().manual_seed(seed)
        n = len(self.actor_params) // 2
        with torch.no_grad():
            for group, head_gain in ((self.actor_params, 0.01), (self.critic_params, 1.0)):
                for i in range(n):
                    w, b = group[2 * i], group[2 * i + 1]
                    gain = head_gain if i == n - 1 else math.sqrt(2.0)
                    w.copy_(_orthogonal(tuple(w.shape), gain, gen))
                    b.zero_()

    @staticmethod
    def _mlp(x, params, final_tanh=False):
        n = len(params) // 2
        for i in range(n):
            x = F.linear(x, params[2 * i], params[2 * i + 1])
            if i < n - 1:
                x = torch.tanh(x)
        return torch.tanh(x) if final_tanh else x

    def actor(self, obs):
        out = self._mlp(obs, self.actor_params)
        return out if self.discrete else torch.tanh(out)

    def critic(self, obs):
        return self._mlp(obs, self.critic_params).squeeze(-1)

    def forward(self, obs):
        return self.actor(obs), self.critic(obs)

    def gaussian_logprob(self, mean, act):
        var = self.gaussian_std ** 2
        return (-0.5 * ((act - mean) ** 2 / var + math.log(2.0 * math.pi * var))).sum(-1)
