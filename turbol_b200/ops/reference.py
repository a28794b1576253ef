"""Plain PyTorch (fp32, CPU-friendly) restatements of every kernel's math.

These are the oracles the kernel tests compare against and the code path CPU
tensors take.  They are written for clarity, not speed.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def philox4x32_10(seed: int, c0: int, c1: int, c2: int, c3: int = 0):
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): the four output words
    for key ``seed`` (64-bit) and counter (c0, c1, c2, c3), as the device and
    host generators compute them."""
    m0, m1, w0, w1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
    mask = 0xFFFFFFFF
    c = [c0 & mask, c1 & mask, c2 & mask, c3 & mask]
    k0, k1 = seed & mask, (seed >> 32) & mask
    for _ in range(10):
        p0, p1 = m0 * c[0], m1 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k0) & mask, p1 & mask, ((p0 >> 32) ^ c[3] ^ k1) & mask, p0 & mask]
        k0, k1 = (k0 + w0) & mask, (k1 + w1) & mask
    return c


def gae(rewards, values, dones, gamma: float = 0.99, lam: float = 0.95):
    """GAE over [T, N] (values [T+1, N]); recurrence of the reference's
    turbol_vllm/src/cuda/gae.cu:31-44."""
    T = rewards.shape[0]
    dt = torch.promote_types(rewards.dtype, torch.float32)
    adv = torch.zeros_like(rewards, dtype=dt)
    last = torch.zeros_like(rewards[0], dtype=dt)
    for t in range(T - 1, -1, -1):
        nd = 1.0 - dones[t].float()
        delta = rewards[t] + gamma * nd * values[t + 1] - values[t]
        last = delta + gamma * lam * nd * last
        adv[t] = last
    return adv, adv + values[:T]


def grpo_advantage(rewards, group_size: int, eps: float = 1e-4, scale_by_std: bool = True):
    r = rewards.float().view(-1, group_size)
    mean = r.mean(1, keepdim=True)
    std = r.std(1, keepdim=True, unbiased=True) if group_size > 1 else torch.zeros_like(mean)
    a = r - mean
    if scale_by_std:
        a = a / (std + eps)
    return a.reshape(-1)


def ppo_categorical_loss(logits, value, act, old_logp, adv, ret, clip=0.2, vf_coef=0.5, ent_coef=0.0,
                         old_value=None, vclip=0.0):
    """Returns (loss, stats) for the clipped-surrogate PPO objective."""
    logp_all = F.log_softmax(logits.float(), -1)
    logp = logp_all.gather(1, act.long().view(-1, 1)).squeeze(1)
    ratio = torch.exp(logp - old_logp)
    pg = -torch.min(ratio * adv, ratio.clamp(1 - clip, 1 + clip) * adv)
    if vclip > 0 and old_value is not None:
        vc = old_value + (value - old_value).clamp(-vclip, vclip)
        vl = 0.5 * torch.max((value - ret) ** 2, (vc - ret) ** 2)
    else:
        vl = 0.5 * (value - ret) ** 2
    ent = -(logp_all.exp() * logp_all).sum(-1)
    loss = pg.mean() + vf_coef * vl.mean() - ent_coef * ent.mean()
    with torch.no_grad():
        stats = torch.stack([pg.sum(), vl.sum(), ent.sum(), ((ratio - 1) - (logp - old_logp)).sum(),
                             ((ratio - 1).abs() > clip).float().sum(), torch.tensor(float(len(act)))])
    return loss, stats


def adam_step(p, g, m, v, step, lr=3e-4, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, grad_scale=1.0):
    g = g * grad_scale
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
    p.sub_(lr * ((m / bc1) / ((v / bc2).sqrt() + eps) + wd * p))
    return p


def fnv1a_reward(ids, lengths=None):
    out = []
    ids = ids.to(torch.int64).cpu()
    for i in range(ids.shape[0]):
        L = int(lengths[i]) if lengths is not None else ids.shape[1]
        h = 0xcbf29ce484222325
        for t in range(min(L, ids.shape[1])):
            w = int(ids[i, t]) & 0xFFFFFFFF
            for _ in range(4):
                h ^= w & 0xFF
                h = (h * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
                w >>= 8
        out.append((h % 1000) / 1000.0)
    return torch.tensor(out, dtype=torch.float32)


def cartpole_step(state, action, gravity=9.8, masscart=1.0, masspole=0.1, length=0.5, force_mag=10.0, tau=0.02,
                  x_threshold=2.4, theta_threshold=12 * 2 * math.pi / 360):
    """One Euler step of the cart-pole equations; returns (next_state, terminated)."""
    x, x_dot, th, th_dot = state.unbind(-1)
    total = masscart + masspole
    pml = masspole * length
    force = torch.where(action == 1, torch.full_like(x, force_mag), torch.full_like(x, -force_mag))
    c, s = torch.cos(th), torch.sin(th)
    temp = (force + pml * th_dot ** 2 * s) / total
    th_acc = (gravity * s - c * temp) / (length * (4.0 / 3.0 - masspole * c ** 2 / total))
    x_acc = temp - pml * th_acc * c / total
    nx = torch.stack([x + tau * x_dot, x_dot + tau * x_acc, th + tau * th_dot, th_dot + tau * th_acc], -1)
    term = (nx[..., 0].abs() > x_threshold) | (nx[..., 2].abs() > theta_threshold)
    return nx, term


def rmsnorm(x, w, eps=1e-6):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float())


def rope(x, pos, theta=1e4):
    """Rotate-half RoPE on the last dim of x [..., S, H, D] with positions [S]."""
    D = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float64, device=x.device) / D))
    ang = pos.to(torch.float64)[:, None] * inv[None, :]
    cos = torch.cos(ang).float()[:, None, :]
    sin = torch.sin(ang).float()[:, None, :]
    x1, x2 = x.float()[..., : D // 2], x.float()[..., D // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)


def causal_attention(q, k, v, scale=None):
    """q [B, S, Hq, D], k/v [B, S, Hk, D] (GQA) -> [B, S, Hq, D] fp32."""
    B, S, Hq, D = q.shape
    Hk = k.shape[2]
    rep = Hq // Hk
    qf, kf, vf = q.float(), k.float().repeat_interleave(rep, 2), v.float().repeat_interleave(rep, 2)
    s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * (scale or 1.0 / math.sqrt(D))
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device).tril()
    s = s.masked_fill(~mask, float("-inf"))
    p = s.softmax(-1)
    return torch.einsum("bhqk,bkhd->bqhd", p, vf)


def lm_forward_ref(model, ids, params=None):
    """fp32 forward of a DecoderLM (all layers, embed and head) from its bf16
    weights; returns logits [B, T, V].  ``params`` (name -> tensor) overrides the
    weights, e.g. with leaf tensors for autograd."""
    cfg = model.cfg
    P = params if params is not None else {n: model.s[n].float() for n in model.offsets}
    if params is None and model.flat is not None:
        for n in P:
            if n.endswith(("ln1", "ln2", "norm", "bqkv")):
                P[n] = model.p[n].float()
    B, T = ids.shape
    H, D, F = cfg.hidden, cfg.head_dim, cfg.ffn
    x = P["embed"][ids.long()]
    pos = torch.arange(T, device=ids.device)
    for i in model.layers:
        p = f"l{i}."
        h = rmsnorm(x, P[p + "ln1"], cfg.rms_eps)
        qkv = h @ P[p + "wqkv"].t()
        if cfg.qkv_bias:
            qkv = qkv + P[p + "bqkv"]
        q = qkv[..., : cfg.q_dim].view(B, T, cfg.n_heads, D)
        k = qkv[..., cfg.q_dim:cfg.q_dim + cfg.kv_dim].view(B, T, cfg.n_kv_heads, D)
        v = qkv[..., cfg.q_dim + cfg.kv_dim:].view(B, T, cfg.n_kv_heads, D)
        q, k = rope(q, pos, cfg.rope_theta), rope(k, pos, cfg.rope_theta)
        a = causal_attention(q, k, v).reshape(B, T, cfg.q_dim)
        x = x + a @ P[p + "wo"].t()
        h = rmsnorm(x, P[p + "ln2"], cfg.rms_eps)
        gu = h @ P[p + "wgu"].t()
        act = torch.nn.functional.silu(gu[..., 0::2]) * gu[..., 1::2]
        x = x + act @ P[p + "wdown"].t()
    h = rmsnorm(x, P["norm"], cfg.rms_eps)
    W = P["embed"] if cfg.tie_embeddings else P["lm_head"]
    return h @ W.t()


def ppo_token_loss(lp, old_lp, adv, v, old_v, ret, clip=0.2, vclip=0.2, vf_coef=0.1, norm=1.0):
    """Clipped PPO policy loss + clipped value loss per token (the oracle of
    the ``ppo_token_loss`` kernel).  Returns (loss, d loss / d lp,
    d loss / d v, stats [pg * norm, vf * norm, clipped tokens, tokens])."""
    lp_t = lp.detach().float().clone().requires_grad_()
    v_t = v.detach().float().clone().requires_grad_()
    with torch.enable_grad():
        ratio = torch.exp(lp_t - old_lp.float())
        pg = -torch.min(ratio * adv, torch.clamp(ratio, 1 - clip, 1 + clip) * adv)
        v_clip = old_v + torch.clamp(v_t - old_v, -vclip, vclip)
        vf = 0.5 * torch.max((v_t - ret) ** 2, (v_clip - ret) ** 2)
        loss = (pg.sum() + vf_coef * vf.sum()) * norm
        loss.backward()
    stats = torch.stack([pg.detach().sum() * norm, vf.detach().sum() * norm,
                         ((ratio.detach() - 1).abs() > clip).float().sum(),
                         torch.tensor(float(lp.numel()), device=lp.device)])
    return loss.detach(), lp_t.grad, v_t.grad, stats
