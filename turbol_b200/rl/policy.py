"""PolicyEngine: actor-critic policy with the reference's API.

Reference: turbol_vllm/include/turbol/policy/policy_engine.hpp:26-54 and
src/policy/policy_engine.cpp:23-138 — a linear Gaussian actor
``mean = tanh(W obs + b)`` with fixed std 0.5, a linear critic, Adam at 1e-3,
``forward(obs, action, logprob)`` / ``get_value(obs, value)`` with
out-parameters and ``update(batch)`` on rows ``[obs | act | adv | ret]``.

Here:
  * the default (``hidden=()``, ``discrete=False``) is that same linear
    Gaussian actor-critic, so reference scripts behave the same;
  * ``hidden=(64, 64)`` etc. gives MLPs, ``discrete=True`` a categorical policy;
  * ``update`` applies the PPO clipped objective when the batch carries the
    behaviour log-prob as an extra column (``[obs | act | adv | ret | old_logp]``);
    without it the ratio is 1 and the gradient equals the reference's
    policy-gradient loss;
  * parameters live in one flat buffer updated by the fused Adam kernel;
  * on a GPU the reference's model (linear Gaussian, ``hidden=()``) acts and
    computes its gradient in one fused kernel each (``lin_gauss_act`` /
    ``lin_gauss_grad``: Philox noise, clipped-PPO + value loss, block-reduced
    parameter gradients), so a step is four launches instead of an autograd
    graph; on the CPU the same passes and Adam run as host loops in the core
    (``lin_gauss_act_host`` / ``lin_gauss_grad_host`` / ``adam_host``);
  * ``forward(obs)`` without out-parameters returns ``(action, logprob)``,
    the form the reference README documents (README.md:149).
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch
import torch.nn.functional as F

from .._native import core as _core
from ..models.mlp import ActorCritic
from ..ops.rl import FusedAdam


def _as_torch(x):
    if isinstance(x, torch.Tensor):
        return x
    if hasattr(x, "torch"):
        return x.torch()
    return torch.as_tensor(x)


class PolicyEngine:
    def __init__(self, obs_dim: int = 4, act_dim: int = 2, device: str = "cpu", hidden: Sequence[int] = (),
                 discrete: bool = False, lr: float = 1e-3, clip: float = 0.2, vf_coef: float = 0.5,
                 ent_coef: float = 0.0, seed: int = 0, std: float = 0.5):
        self.obs_dim, self.act_dim = obs_dim, act_dim
        from ..utils.device import parse_device
        self.device = parse_device(device)
        self.hidden, self.discrete, self.lr = tuple(hidden), discrete, lr
        self.clip, self.vf_coef, self.ent_coef, self.seed, self.std = clip, vf_coef, ent_coef, seed, std
        self.net: Optional[ActorCritic] = None
        self.opt: Optional[FusedAdam] = None
        self._gen = None
        self._calls = 0  # Philox counter of the fused sampler

    # -------------------------------------------------------------- lifecycle
    def initialize(self):
        Status = _core().Status
        self.net = ActorCritic(self.obs_dim, self.act_dim, self.hidden, self.discrete, self.device, self.seed,
                               gaussian_std=self.std)
        self.opt = FusedAdam(self.net.fp.flat, self.net.fp.grad, lr=self.lr)
        self._gen = torch.Generator(device=self.device).manual_seed(self.seed + 12345)
        return Status()

    def _check(self):
        if self.net is None:
            raise RuntimeError("PolicyEngine not initialized")

    def _fused(self) -> bool:
        """The fused kernels serve the linear Gaussian model on a GPU."""
        return (self.device.type == "cuda" and not self.hidden and not self.discrete and self.obs_dim <= 64
                and self.act_dim <= 16)

    def _host_fused(self) -> bool:
        """On the CPU the same model runs the host versions of those passes
        (``lin_gauss_act_host`` / ``lin_gauss_grad_host``): plain loops, no
        per-operator dispatch for the small tensors."""
        return self.device.type == "cpu" and not self.hidden and not self.discrete

    # -------------------------------------------------------------- acting
    @torch.no_grad()
    def act(self, obs: torch.Tensor):
        """Returns (action, logprob) for obs [N, obs_dim]."""
        self._check()
        obs = _as_torch(obs).to(self.device, torch.float32)
        if self.discrete:
            logits = self.net.actor(obs)
            logp_all = F.log_softmax(logits, -1)
            a = torch.multinomial(logp_all.exp(), 1, generator=self._gen).squeeze(1)
            return a.to(torch.int32), logp_all.gather(1, a[:, None]).squeeze(1)
        if self._fused() or self._host_fused():
            x = obs.reshape(-1, self.obs_dim).contiguous()
            a = torch.empty(x.shape[0], self.act_dim, device=self.device)
            lp = torch.empty(x.shape[0], device=self.device)
            self._calls += 1
            if self._fused():
                from .._native import ops as _ops
                _ops().lin_gauss_act(x, self.net.fp.flat, a, lp, self.obs_dim, self.act_dim, self.std,
                                     self.seed + 12345, self._calls & 0xFFFFFFFF)
            else:
                _core().lin_gauss_act_host(x, self.net.fp.flat.detach(), a, lp, self.obs_dim, self.act_dim, self.std,
                                           self.seed + 12345, self._calls & 0xFFFFFFFF)
            return a, lp
        mean = self.net.actor(obs)
        noise = torch.randn(mean.shape, device=self.device, generator=self._gen)
        a = (mean + self.std * noise).clamp(-1.0, 1.0)
        return a, self.net.gaussian_logprob(mean, a)

    def forward(self, observation, action=None, logprob=None):
        a, lp = self.act(observation)
        if action is None and logprob is None:
            return a, lp
        T = _core().Tensor
        action.set_(a.float().contiguous() if not self.discrete else a)
        logprob.set_(lp.contiguous())
        return _core().Status()

    @torch.no_grad()
    def value(self, obs):
        self._check()
        return self.net.critic(_as_torch(obs).to(self.device, torch.float32))

    def get_value(self, observation, value=None):
        v = self.value(observation)
        if value is None:
            return v
        value.set_(v.contiguous())
        return _core().Status()

    # -------------------------------------------------------------- learning
    def update(self, batch):
        """One gradient step on rows [obs | act | adv | ret (| old_logp)].

        ``act`` is ``act_dim`` wide for the Gaussian policy and 1 wide (the
        action index) for the categorical one."""
        self._check()
        b = _as_torch(batch).to(self.device, torch.float32)
        aw = 1 if self.discrete else self.act_dim
        row = self.obs_dim + aw + 2
        if b.numel() % row != 0 and b.numel() % (row + 1) != 0:
            raise ValueError("batch size must be a multiple of obs+act+adv+ret(+old_logp)")
        has_old = b.dim() == 2 and b.shape[1] == row + 1
        b = b.reshape(-1, row + 1 if has_old else row)
        if self._fused():
            from .._native import ops as _ops
            self.net.fp.grad.zero_()
            _ops().lin_gauss_grad(b.contiguous(), self.net.fp.flat, self.net.fp.grad, self.obs_dim, self.act_dim,
                                  self.std, self.clip, self.vf_coef, has_old)
            self.opt.step()
            return _core().Status()
        if self._host_fused():
            g = self.net.fp.grad
            g.zero_()
            _core().lin_gauss_grad_host(b.contiguous(), self.net.fp.flat.detach(), g, self.obs_dim, self.act_dim,
                                        self.std, self.clip, self.vf_coef, has_old)
            self.opt.step()
            return _core().Status()
        obs = b[:, : self.obs_dim]
        act = b[:, self.obs_dim:self.obs_dim + aw]
        adv = b[:, self.obs_dim + aw]
        ret = b[:, self.obs_dim + aw + 1]
        self.net.fp.zero_grad()
        if self.discrete:
            logits = self.net.actor(obs)
            logp_all = F.log_softmax(logits, -1)
            logp = logp_all.gather(1, act.long()).squeeze(1)
            ent = -(logp_all.exp() * logp_all).sum(-1).mean()
        else:
            mean = self.net.actor(obs)
            logp = self.net.gaussian_logprob(mean, act)
            ent = torch.zeros((), device=self.device)
        old = b[:, -1] if has_old else logp.detach()
        ratio = torch.exp(logp - old)
        pg = -torch.min(ratio * adv, ratio.clamp(1 - self.clip, 1 + self.clip) * adv).mean()
        v = self.net.critic(obs)
        loss = pg + self.vf_coef * F.mse_loss(v, ret) - self.ent_coef * ent
        loss.backward()
        self.opt.step()
        return _core().Status()

    # -------------------------------------------------------------- state
    def state_dict(self):
        self._check()
        return {"net": self.net.state_dict(), "optim": self.opt.state_dict(),
                "config": {"obs_dim": self.obs_dim, "act_dim": self.act_dim, "hidden": list(self.hidden),
                           "discrete": self.discrete, "lr": self.lr}}

    def load_state_dict(self, sd):
        self._check()
        with torch.no_grad():
            self.net.load_state_dict(sd["net"])
        self.opt.load_state_dict(sd["optim"])
