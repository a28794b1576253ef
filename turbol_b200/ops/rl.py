"""RL op wrappers: CUDA tensors go to the sm_100a kernels, CPU tensors to the
reference math in :mod:`turbol_b200.ops.reference`."""
from __future__ import annotations

import torch

from .._native import core as _core, ops as _ops
from . import reference as ref


def gae(rewards, values, dones, gamma: float = 0.99, lam: float = 0.95, stats=None, scratch=None, out=None):
    """Returns (advantages, returns) for rewards/dones [T, N], values [T+1, N].

    ``stats`` (float64 [2]) accumulates sum and sum of squares of the
    advantages; ``scratch`` is the chunk-map workspace (allocated here if
    needed and not given)."""
    if not rewards.is_cuda:
        if rewards.dtype == torch.float32 and values.dtype == torch.float32 and rewards.dim() == 2:
            # one backward sweep in the core (the recurrence of ref.gae)
            adv, ret = out if out is not None else (torch.empty_like(rewards), torch.empty_like(rewards))
            d = dones if dones.dtype in (torch.bool, torch.uint8) else dones.to(torch.uint8)
            _core().gae_host(rewards.contiguous(), values.contiguous(), d.contiguous(), adv, ret, stats, gamma, lam)
            return adv, ret
        return ref.gae(rewards, values, dones, gamma, lam)
    adv, ret = out if out is not None else (torch.empty_like(rewards), torch.empty_like(rewards))
    d = dones if dones.dtype in (torch.bool, torch.uint8) else dones.to(torch.uint8)
    _ops().gae(rewards.contiguous(), values.contiguous(), d.contiguous(), adv, ret, stats, scratch, gamma, lam)
    return adv, ret


def grpo_advantage(rewards, group_size: int, eps: float = 1e-4, scale_by_std: bool = True):
    if not rewards.is_cuda:
        return ref.grpo_advantage(rewards, group_size, eps, scale_by_std)
    return _ops().grpo_advantage(rewards.float().contiguous(), group_size, eps, scale_by_std)


class _PPOCategoricalLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, value, act, old_logp, adv, ret, old_value, stats, clip, vclip, vf_coef, ent_coef):
        dlogits = torch.empty_like(logits)
        dvalue = torch.empty_like(value)
        _ops().ppo_loss(logits, value, act, old_logp, adv, ret, old_value, dlogits, dvalue, stats, clip, vclip,
                        vf_coef, ent_coef)
        ctx.save_for_backward(dlogits, dvalue)
        # The scalar loss value is carried by `stats`; the returned tensor only
        # anchors the graph (its gradient is what the kernel computed).
        return logits.new_zeros(())

    @staticmethod
    def backward(ctx, g):
        dlogits, dvalue = ctx.saved_tensors
        return dlogits * g, dvalue * g, None, None, None, None, None, None, None, None, None, None


def ppo_categorical_loss(logits, value, act, old_logp, adv, ret, clip=0.2, vf_coef=0.5, ent_coef=0.0,
                         old_value=None, vclip=0.0, stats=None):
    """Clipped-surrogate PPO loss for a categorical policy.

    CUDA: one fused forward+backward kernel; the returned scalar is a graph
    anchor (0-valued) whose backward delivers the exact gradients, and the loss
    terms are accumulated into ``stats`` = [pg_sum, v_sum, ent_sum, kl_sum,
    clipfrac_sum, count].  CPU: the reference expression (real loss value)."""
    if not logits.is_cuda:
        loss, st = ref.ppo_categorical_loss(logits, value, act, old_logp, adv, ret, clip, vf_coef, ent_coef,
                                            old_value, vclip)
        if stats is not None:
            stats[: st.numel()] += st.to(stats)
        return loss
    return _PPOCategoricalLoss.apply(logits.float().contiguous(), value.float().contiguous(), act, old_logp, adv,
                                     ret, old_value, stats, clip, vclip, vf_coef, ent_coef)


class FusedAdam:
    """Adam over one flat fp32 buffer: one launch per step, step count on the
    device (so the step can be captured in a CUDA graph), optional bf16 shadow
    of the weights written in the same pass."""

    def __init__(self, flat_param, flat_grad, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                 max_grad_norm=0.0, bf16_shadow=False, shadow=None):
        self.p, self.g = flat_param, flat_grad
        self.m = torch.zeros_like(flat_param)
        self.v = torch.zeros_like(flat_param)
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.max_grad_norm = max_grad_norm
        self.step_t = torch.zeros(1, dtype=torch.int64, device=flat_param.device)
        if shadow is not None:
            self.shadow = shadow
        else:
            self.shadow = torch.empty_like(flat_param, dtype=torch.bfloat16) if bf16_shadow else None
        self.gnorm = torch.zeros(1, dtype=torch.float32, device=flat_param.device) if max_grad_norm > 0 else None
        self._host_step = 0

    def step(self, grad_scale: float = 1.0):
        if not self.p.is_cuda:
            self._host_step += 1
            p = self.p.data
            if all(t.dtype == torch.float32 and t.is_contiguous() for t in (p, self.g, self.m, self.v)):
                # one pass in the core (the same update as ref.adam_step)
                _core().adam_host(p, self.g, self.m, self.v, self._host_step, self.lr, self.betas[0], self.betas[1],
                                  self.eps, self.wd, grad_scale)
            else:
                ref.adam_step(p, self.g, self.m, self.v, self._host_step, self.lr, self.betas[0], self.betas[1],
                              self.eps, self.wd, grad_scale)
            if self.shadow is not None:
                self.shadow.copy_(self.p)
            return
        o = _ops()
        if self.gnorm is not None:
            self.gnorm.zero_()
            o.sumsq(self.g, self.gnorm)
        o.adam(self.p.data, self.g, self.m, self.v, self.shadow, self.lr, self.betas[0], self.betas[1], self.eps,
               self.wd, grad_scale, self.max_grad_norm, self.step_t, 0, self.gnorm)
        o.counter_add(self.step_t, 1)

    def state_dict(self):
        return {"m": self.m, "v": self.v, "step": self.step_t.clone() if self.p.is_cuda else self._host_step,
                "lr": self.lr, "betas": self.betas, "eps": self.eps, "wd": self.wd}

    def load_state_dict(self, sd):
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        if self.p.is_cuda:
            self.step_t.copy_(torch.as_tensor(sd["step"]).to(self.step_t))
        else:
            self._host_step = int(sd["step"])


def hash_reward(token_ids, lengths=None):
    if not token_ids.is_cuda:
        return ref.fnv1a_reward(token_ids, lengths)
    ids = token_ids.to(torch.int32).contiguous()
    lens = (lengths if lengths is not None else torch.full((ids.shape[0],), ids.shape[1], device=ids.device))
    return _ops().hash_reward(ids, lens.to(torch.int32).contiguous())
