#!/usr/bin/env python
"""Labelled BASELINE (not the product): the two headline workloads written the
plain way, PyTorch eager + cuBLAS/cuDNN-backed torch ops + torch.distributed
NCCL, with the same math, shapes and batch as this framework's bench.

  python benchmarks/baseline_eager.py ppo  [--steps K] [--warmup W]
  python benchmarks/baseline_eager.py grpo [--steps K] [--warmup W]
  torchrun --nproc-per-node N benchmarks/baseline_eager.py {ppo,grpo} --gpus N

ppo   65,536 CartPole envs per GPU (torch tensor ops, auto-reset), rollout 128,
      actor and critic MLPs 4-256-256-{2,1} tanh (nn.Sequential, bf16 autocast,
      fp32 weights), GAE (gamma 0.99, lambda 0.95) as a Python loop of tensor
      ops, 4 epochs of minibatch 32,768 with clip 0.2, value coefficient 0.5 and
      torch.optim.Adam(3e-4); several GPUs: DistributedDataParallel (NCCL
      all-reduce of gradient buckets overlapped with backward).
grpo  decoder with the 1.5B shape (28 layers, hidden 1536, 12 q / 2 kv heads,
      head_dim 128, SwiGLU 8960, vocab 151,936, RoPE 1e6, tied embedding,
      QKV bias), random init; 64 prompts x 8 samples, 256 + 512 tokens,
      temperature 1.0; rollout = prefill + a KV-cache decode loop with
      F.scaled_dot_product_attention and torch.multinomial; hash reward (FNV-1a
      64 of the response ids mod 1000 / 1000), group-normalized advantages,
      reference log-probs under a frozen copy, clipped GRPO loss with the k3 KL
      (coefficient 0.04) in micro-batches of 8 sequences, one AdamW step
      (lr 1e-6, betas 0.9 / 0.95); several GPUs: DDP over the same global batch
      (64 prompts per 2 GPUs, the per-GPU work of a TP2 layout).

Every step is timed with CUDA events on the device (max over ranks).  One JSON
line per run, with "impl": "eager-baseline".  The reference itself has no PPO
or GRPO training path (its examples step a linear env with random actions and
echo prompts: turbol_vllm/examples/py/ppo_example.py:146-210,
grpo_example.py:124-151), so this is the same-config anchor for both halves
of the headline metric.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("workload", choices=["ppo", "grpo"])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None)
    p.add_argument("--warmup", type=int, default=None)
    p.add_argument("--num-envs", type=int, default=65536)
    p.add_argument("--prompts", type=int, default=None, help="GRPO prompts per GPU (default: 64 on one GPU, "
                                                             "32 on several: the global batch of a TP2 layout)")
    return p.parse_args()


def setup(n):
    rank, world, local = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(
        os.environ.get("LOCAL_RANK", 0))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sync(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


# ============================================================================ PPO
class CartPole:
    """Vectorized CartPole (the classic equations, Euler step dt 0.02, force
    +-10), auto-reset to U[-0.05, 0.05] at |x| > 2.4, |theta| > 12 deg or 500 steps."""

    def __init__(self, n, device, gen):
        self.n, self.dev, self.gen = n, device, gen
        self.s = (torch.rand(n, 4, device=device, generator=gen) - 0.5) * 0.1
        self.t = torch.zeros(n, device=device, dtype=torch.int32)

    def step(self, a):
        x, xd, th, thd = self.s.unbind(1)
        force = torch.where(a == 1, 10.0, -10.0)
        ct, st = torch.cos(th), torch.sin(th)
        mp, mt, l = 0.1, 1.1, 0.5
        temp = (force + mp * l * thd * thd * st) / mt
        tha = (9.8 * st - ct * temp) / (l * (4.0 / 3.0 - mp * ct * ct / mt))
        xa = temp - mp * l * tha * ct / mt
        x, xd, th, thd = x + 0.02 * xd, xd + 0.02 * xa, th + 0.02 * thd, thd + 0.02 * tha
        self.t += 1
        term = (x.abs() > 2.4) | (th.abs() > 12 * 2 * math.pi / 360)
        done = term | (self.t >= 500)
        ns = torch.stack([x, xd, th, thd], 1)
        fresh = (torch.rand(self.n, 4, device=self.dev, generator=self.gen) - 0.5) * 0.1
        self.s = torch.where(done[:, None], fresh, ns)
        self.t = torch.where(done, torch.zeros_like(self.t), self.t)
        return self.s, torch.ones(self.n, device=self.dev), done


class ActorCritic(nn.Module):
    def __init__(self, hidden=256):
        super().__init__()
        self.actor = nn.Sequential(nn.Linear(4, hidden), nn.Tanh(), nn.Linear(hidden, hidden), nn.Tanh(),
                                   nn.Linear(hidden, 2))
        self.critic = nn.Sequential(nn.Linear(4, hidden), nn.Tanh(), nn.Linear(hidden, hidden), nn.Tanh(),
                                    nn.Linear(hidden, 1))
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.orthogonal_(m.weight, math.sqrt(2))
                nn.init.zeros_(m.bias)

    def forward(self, obs):
        return self.actor(obs), self.critic(obs).squeeze(-1)


def run_ppo(args, rank, world, local):
    dev = torch.device("cuda", local)
    N, T, MB, EPOCHS = args.num_envs, 128, 32768, 4
    gen = torch.Generator(device=dev).manual_seed(17 + 104729 * rank)
    torch.manual_seed(1)
    env = CartPole(N, dev, gen)
    net = ActorCritic().to(dev)
    model = net
    if world > 1:
        model = nn.parallel.DistributedDataParallel(net, device_ids=[local])
    opt = torch.optim.Adam(net.parameters(), lr=3e-4)
    obs_b = torch.zeros(T, N, 4, device=dev)
    act_b = torch.zeros(T, N, device=dev, dtype=torch.long)
    logp_b = torch.zeros(T, N, device=dev)
    val_b = torch.zeros(T + 1, N, device=dev)
    rew_b = torch.zeros(T, N, device=dev)
    done_b = torch.zeros(T, N, device=dev)
    ret_sum = torch.zeros(N, device=dev)
    ep_stats = torch.zeros(2, device=dev)

    def iteration():
        obs = env.s
        with torch.no_grad(), torch.autocast("cuda", torch.bfloat16):
            for t in range(T):
                logits, v = net(obs)
                probs = torch.softmax(logits.float(), -1)
                a = torch.multinomial(probs, 1, generator=gen).squeeze(1)
                obs_b[t] = obs
                act_b[t] = a
                logp_b[t] = torch.log(probs.gather(1, a[:, None]).squeeze(1))
                val_b[t] = v.float()
                obs, r, d = env.step(a)
                rew_b[t] = r
                done_b[t] = d.float()
                ret_sum.add_(r)
                ep_stats[0] += (ret_sum * d).sum()
                ep_stats[1] += d.sum()
                ret_sum.mul_(1.0 - d.float())
            val_b[T] = net(obs)[1].float()
        adv = torch.zeros(T, N, device=dev)
        last = torch.zeros(N, device=dev)
        for t in reversed(range(T)):  # GAE
            nd = 1.0 - done_b[t]
            delta = rew_b[t] + 0.99 * val_b[t + 1] * nd - val_b[t]
            last = delta + 0.99 * 0.95 * nd * last
            adv[t] = last
        ret = adv + val_b[:T]
        fo, fa, fl, fadv, fret = (obs_b.view(-1, 4), act_b.view(-1), logp_b.view(-1), adv.view(-1), ret.view(-1))
        B = T * N
        for _ in range(EPOCHS):
            perm = torch.randperm(B, device=dev, generator=gen)
            for i in range(0, B, MB):
                idx = perm[i:i + MB]
                a_adv = fadv[idx]
                a_adv = (a_adv - a_adv.mean()) / (a_adv.std() + 1e-8)
                with torch.autocast("cuda", torch.bfloat16):
                    logits, v = model(fo[idx])
                lp = torch.log_softmax(logits.float(), -1).gather(1, fa[idx][:, None]).squeeze(1)
                ratio = torch.exp(lp - fl[idx])
                pg = -torch.min(ratio * a_adv, torch.clamp(ratio, 0.8, 1.2) * a_adv).mean()
                vl = 0.5 * ((v.float() - fret[idx]) ** 2).mean()
                opt.zero_grad(set_to_none=False)
                (pg + 0.5 * vl).backward()
                opt.step()

    steps = args.steps if args.steps is not None else 3
    warm = args.warmup if args.warmup is not None else 3
    for _ in range(warm):
        iteration()
    sync(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        iteration()
    e1.record()
    sync(world)
    sec = max_over_ranks(e0.elapsed_time(e1) / 1e3, world)
    mean_ret = float(ep_stats[0] / ep_stats[1].clamp(min=1))
    return {"impl": "eager-baseline", "metric": "PPO env-steps/s (64K envs)", "value": world * N * T * steps / sec,
            "unit": "env-steps/s", "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": sec / steps * 1e3, "dtype": "bf16 autocast, fp32 weights",
            "config": {"model": "CartPole PPO actor-critic MLP 4-256-256-{2,1} tanh", "num_envs_per_gpu": N,
                       "rollout": T, "minibatch": MB, "epochs": EPOCHS,
                       "parallelism": f"ddp{world}" if world > 1 else "dp1"},
            "mean_return": mean_ret, "timing": "CUDA events, max over ranks"}


# ============================================================================ GRPO
class Cfg:
    L, H, HQ, HK, D, FF, V, THETA, EPS = 28, 1536, 12, 2, 128, 8960, 151936, 1e6, 1e-6


def rope(x, cos, sin):
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return x * cos + torch.cat([-x2, x1], -1) * sin


class Block(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.ln1 = nn.Parameter(torch.ones(c.H))
        self.ln2 = nn.Parameter(torch.ones(c.H))
        self.qkv = nn.Linear(c.H, (c.HQ + 2 * c.HK) * c.D, bias=True)
        self.o = nn.Linear(c.HQ * c.D, c.H, bias=False)
        self.gu = nn.Linear(c.H, 2 * c.FF, bias=False)
        self.down = nn.Linear(c.FF, c.H, bias=False)
        self.c = c

    @staticmethod
    def norm(x, w, eps):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w).to(torch.bfloat16)

    def forward(self, x, cos, sin, cache=None, pos=None):
        """x [B, S, H].  cache: (k_cache, v_cache) [B, HK, Lmax, D] and the write
        position pos (decode: S == 1, attends to [0, pos])."""
        c = self.c
        B, S, _ = x.shape
        h = self.norm(x, self.ln1, c.EPS)
        q, k, v = self.qkv(h).split([c.HQ * c.D, c.HK * c.D, c.HK * c.D], -1)
        q = rope(q.view(B, S, c.HQ, c.D).transpose(1, 2), cos, sin)
        k = rope(k.view(B, S, c.HK, c.D).transpose(1, 2), cos, sin)
        v = v.view(B, S, c.HK, c.D).transpose(1, 2)
        if cache is None:
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        else:
            kc, vc = cache
            if S > 1:  # prefill into the cache
                kc[:, :, :S] = k
                vc[:, :, :S] = v
                a = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
            else:
                kc[:, :, pos:pos + 1] = k
                vc[:, :, pos:pos + 1] = v
                a = F.scaled_dot_product_attention(q, kc[:, :, :pos + 1], vc[:, :, :pos + 1], enable_gqa=True)
        x = x + self.o(a.transpose(1, 2).reshape(B, S, c.HQ * c.D))
        h = self.norm(x, self.ln2, c.EPS)
        g, u = self.gu(h).chunk(2, -1)
        return x + self.down(F.silu(g) * u)


class EagerLM(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.c = c
        self.embed = nn.Embedding(c.V, c.H)
        self.blocks = nn.ModuleList([Block(c) for _ in range(c.L)])
        self.norm = nn.Parameter(torch.ones(c.H))
        for p in self.parameters():
            if p.dim() == 2:
                nn.init.normal_(p, std=0.02)
        for b in self.blocks:
            nn.init.zeros_(b.qkv.bias)
        inv = 1.0 / (c.THETA ** (torch.arange(0, c.D, 2, dtype=torch.float64) / c.D))
        ang = torch.arange(4096, dtype=torch.float64)[:, None] * inv[None, :]
        ang = torch.cat([ang, ang], -1)
        self.register_buffer("cos", torch.cos(ang).float(), persistent=False)
        self.register_buffer("sin", torch.sin(ang).float(), persistent=False)

    def hidden(self, ids, caches=None, pos=None):
        S = ids.shape[1]
        p0 = 0 if pos is None else pos
        cos, sin = self.cos[p0:p0 + S].to(torch.bfloat16), self.sin[p0:p0 + S].to(torch.bfloat16)
        x = self.embed(ids).to(torch.bfloat16)
        for i, b in enumerate(self.blocks):
            x = b(x, cos, sin, None if caches is None else caches[i], pos)
        return Block.norm(x, self.norm, self.c.EPS)

    def logits(self, h):
        return F.linear(h, self.embed.weight.to(torch.bfloat16))

    def forward(self, ids, prompt_len: int):
        """Log-probs [B, S - prompt_len] of the response tokens ids[:, prompt_len:]."""
        S = ids.shape[1]
        h = self.hidden(ids)[:, prompt_len - 1:S - 1]
        logits = self.logits(h).float()
        return torch.log_softmax(logits, -1).gather(2, ids[:, prompt_len:, None]).squeeze(2)


def hash_reward(resp):
    """(FNV-1a 64 over the little-endian bytes of the int32 ids) mod 1000 / 1000."""
    h = torch.full((resp.shape[0],), -3750763034362895579, dtype=torch.int64, device=resp.device)  # 0xcbf29ce484222325
    prime = 0x100000001B3
    w = resp.to(torch.int64) & 0xFFFFFFFF
    for t in range(resp.shape[1]):
        x = w[:, t]
        for _ in range(4):
            h = (h ^ (x & 0xFF)) * prime
            x = x >> 8
    m = torch.remainder(h, 1000)
    m = torch.where(h < 0, torch.remainder(m + 616, 1000), m)  # unsigned value: 2^64 mod 1000 = 616
    return m.float() / 1000.0


def run_grpo(args, rank, world, local):
    dev = torch.device("cuda", local)
    c = Cfg()
    P = args.prompts if args.prompts is not None else (64 if world == 1 else 32)
    G, Lp, Lr, mb = 8, 256, 512, 8
    B, T = P * G, Lp + Lr
    torch.manual_seed(0)
    model = EagerLM(c).to(dev)
    ref = EagerLM(c).to(dev).to(torch.bfloat16)
    ref.load_state_dict({k: v.to(torch.bfloat16) for k, v in model.state_dict().items()})
    ref.requires_grad_(False)
    ddp = nn.parallel.DistributedDataParallel(model, device_ids=[local]) if world > 1 else model
    opt = torch.optim.AdamW(model.parameters(), lr=1e-6, betas=(0.9, 0.95), weight_decay=0.0, fused=True)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    caches = [(torch.empty(B, c.HK, T, c.D, device=dev, dtype=torch.bfloat16),
               torch.empty(B, c.HK, T, c.D, device=dev, dtype=torch.bfloat16)) for _ in range(c.L)]
    step_no = [0]

    @torch.no_grad()
    def rollout(prompts):
        with torch.autocast("cuda", torch.bfloat16):
            pc = [(torch.empty(P, c.HK, T, c.D, device=dev, dtype=torch.bfloat16),
                   torch.empty(P, c.HK, T, c.D, device=dev, dtype=torch.bfloat16)) for _ in range(c.L)]
            h = model.hidden(prompts, pc, 0)[:, -1]
            for (kc, vc), (pk, pv) in zip(caches, pc):  # each prompt's KV to its G samples
                kc[:, :, :Lp] = pk[:, :, :Lp].repeat_interleave(G, 0)
                vc[:, :, :Lp] = pv[:, :, :Lp].repeat_interleave(G, 0)
            del pc
            h = h.repeat_interleave(G, 0)
            toks, lps = [], []
            for t in range(Lr):
                logits = model.logits(h).float()
                probs = torch.softmax(logits, -1)
                tok = torch.multinomial(probs, 1, generator=gen)
                toks.append(tok)
                lps.append(torch.log(probs.gather(1, tok)))
                if t + 1 < Lr:
                    h = model.hidden(tok, caches, Lp + t)[:, -1]
        return torch.cat([prompts.repeat_interleave(G, 0), torch.cat(toks, 1)], 1), torch.cat(lps, 1)

    def step():
        g = torch.Generator(device=dev).manual_seed(step_no[0] * 1000003 + 104729 * rank)
        prompts = torch.randint(0, c.V, (P, Lp), generator=g, device=dev)
        step_no[0] += 1
        seqs, _ = rollout(prompts)
        r = hash_reward(seqs[:, Lp:]).view(P, G)
        adv = ((r - r.mean(1, keepdim=True)) / (r.std(1, keepdim=True) + 1e-4)).view(-1)
        with torch.no_grad(), torch.autocast("cuda", torch.bfloat16):
            ref_lp = torch.cat([ref(seqs[i:i + mb], Lp) for i in range(0, B, mb)])
        opt.zero_grad(set_to_none=False)
        n_mb = B // mb
        for j, i in enumerate(range(0, B, mb)):
            ctx = ddp.no_sync() if (world > 1 and j + 1 < n_mb) else _null()
            with ctx:
                with torch.autocast("cuda", torch.bfloat16):
                    lp = ddp(seqs[i:i + mb], Lp)  # through DDP: its hooks all-reduce on the last micro-batch
                old = lp.detach()
                ratio = torch.exp(lp - old)
                a = adv[i:i + mb, None]
                pg = -torch.min(ratio * a, torch.clamp(ratio, 0.8, 1.2) * a)
                d = ref_lp[i:i + mb] - lp
                kl = torch.exp(d) - d - 1
                loss = ((pg + 0.04 * kl).mean(1)).sum() / B
                loss.backward()
        opt.step()

    steps = args.steps if args.steps is not None else 2
    warm = args.warmup if args.warmup is not None else 3
    for _ in range(warm):
        step()
    times = []
    for _ in range(steps):
        sync(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        torch.cuda.synchronize()
        times.append(max_over_ranks(e0.elapsed_time(e1) / 1e3, world))
    sec = sum(times) / len(times)
    return {"impl": "eager-baseline", "metric": "GRPO train tokens/s/box", "value": world * B * T / sec,
            "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": warm, "s_per_step": sec,
            "dtype": "bf16 autocast, fp32 weights",
            "config": {"model": "qwen2-1.5b-shape decoder (28 layers, hidden 1536, 12q/2kv heads, ffn 8960, "
                                "vocab 151936)", "prompts_per_gpu": P, "group": G, "prompt_len": Lp,
                       "response_len": Lr, "global_batch_sequences": world * B,
                       "parallelism": f"ddp{world}" if world > 1 else "dp1"},
            "timing": "CUDA events around each step, max over ranks"}


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def main():
    args = parse()
    rank, world, local = setup(args.gpus)
    out = run_ppo(args, rank, world, local) if args.workload == "ppo" else run_grpo(args, rank, world, local)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        sync(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
