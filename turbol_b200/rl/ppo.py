"""PPO for vectorized device-resident environments (CartPole).

One training iteration = a rollout of ``rollout_steps`` steps over
``num_envs`` environments, GAE, then ``epochs`` passes of shuffled minibatches
of the clipped-surrogate objective.

GPU path (everything stays on the device, no host round trip per step):
  rollout step   policy MLP forward (bf16 tensor cores under autocast) ->
                 one fused kernel: sample action (Gumbel-max), log-prob, store
                 the transition at row t, step CartPole with auto-reset;
  advantages     one GAE kernel that also accumulates the advantage moments;
  minibatch      gather through an on-device Feistel permutation (fused with
                 advantage normalization) -> hidden layers -> one kernel for
                 the output layer, the clipped loss and the output-layer
                 backward -> weight-gradient GEMMs into one flat gradient
                 buffer -> [data-parallel gradient reduction] -> one fused
                 Adam launch.
The rollout, the advantage pass and one minibatch step are each captured as a
CUDA graph; the minibatch graph is replayed epochs * n_minibatches times and
reads its (epoch, minibatch) position from a device counter.

CPU path: the same algorithm in eager PyTorch with the reference math (used by
the CPU tests and as the oracle for the kernels).

The reference's ppo_example.py (turbol_vllm/examples/py/ppo_example.py:146-210)
steps a linear env with random actions and never runs GAE or a clipped update;
this module is the algorithm its name promises.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Optional

import torch
import torch.nn.functional as F

from .._native import core as _core, ops as _ops
from ..models.mlp import ActorCritic
from ..ops import reference as ref
from ..ops.rl import FusedAdam, gae, ppo_categorical_loss


@dataclass
class PPOConfig:
    num_envs: int = 256
    rollout_steps: int = 32
    hidden: tuple = (64, 64)
    epochs: int = 4
    minibatch_size: int = 64
    lr: float = 3e-4
    gamma: float = 0.99
    lam: float = 0.95
    clip: float = 0.2
    vf_coef: float = 0.5
    ent_coef: float = 0.0
    max_grad_norm: float = 0.0
    norm_adv: bool = True
    seed: int = 1
    compute_dtype: str = "bf16"  # "bf16" (tensor cores, fp32 master weights) or "fp32"
    cuda_graphs: bool = True
    env: str = "cartpole"
    # CPU device: intra-op threads during an iteration (0 = automatic: the
    # process's setting for the core's host rollout / update, which split a
    # large minibatch over at most that many threads and keep a small one on
    # the calling thread; for the torch-op path, one thread when the
    # minibatch's matrix products are small, where forking the thread pool
    # per operator costs more than the arithmetic); the process's setting is
    # restored after the iteration
    cpu_threads: int = 0

    @property
    def batch(self) -> int:
        return self.num_envs * self.rollout_steps

    @property
    def n_minibatches(self) -> int:
        return max(1, self.batch // self.minibatch_size)


class PPOTrainer:
    """PPO trainer; ``grad_sync`` (optional) reduces the flat gradient across
    data-parallel ranks in place and returns the scale Adam applies."""

    def __init__(self, cfg: PPOConfig, device="cuda:0", grad_sync: Optional[Callable] = None, rank: int = 0,
                 dp: str = "none", group=None):
        """dp: "none"; "nccl" (NCCL all-reduce of the gradient + local fused
        Adam); "fused" (one NVLink peer-memory kernel: gradient reduce-scatter,
        sharded Adam, weight all-gather)."""
        self.cfg, self.rank, self.dp, self.group = cfg, rank, dp, group
        if dp == "fused" and not (device.startswith("cuda") if isinstance(device, str) else device.type == "cuda"):
            raise ValueError("the fused data-parallel step needs CUDA devices")
        if dp == "nccl" and grad_sync is None:
            from ..parallel.dp import NcclGradSync

            grad_sync = NcclGradSync(group)
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        C = _core()
        T, N = cfg.rollout_steps, cfg.num_envs
        if cfg.batch % cfg.minibatch_size != 0:
            raise ValueError("num_envs * rollout_steps must be a multiple of minibatch_size")
        dev = str(self.device) if self.cuda else "cpu"
        self.env = C.GPUEnvironment(N, 4, 2, dev, "cartpole", seed=cfg.seed * 7919 + rank * 104729 + 17)
        # tensor-core path: bf16 GEMMs with fused epilogues and a hand-written
        # backward; otherwise PyTorch autograd (CPU, fp32 or unequal hidden sizes)
        self.fused = (self.cuda and cfg.compute_dtype == "bf16" and len(cfg.hidden) == 2
                      and cfg.hidden[0] == cfg.hidden[1] and cfg.hidden[0] % 64 == 0)
        if self.fused:
            from ..models.fused_mlp import FusedActorCritic

            self.net = FusedActorCritic(4, 2, cfg.hidden, device=self.device, seed=cfg.seed)
            self.policy = None
            self.flat, self.flat_grad = self.net.flat, self.net.grad
            if dp == "fused":
                from ..parallel.peer import FusedDataParallelAdam

                self.opt = FusedDataParallelAdam(self.net.numel, group, lr=cfg.lr)
                self.net.rebind_storage(self.opt.param, self.opt.grad, self.opt.shadow)
                self.opt.broadcast_params(0)
                self.flat, self.flat_grad = self.net.flat, self.net.grad
            else:
                self.opt = FusedAdam(self.net.flat, self.net.grad, lr=cfg.lr, max_grad_norm=cfg.max_grad_norm,
                                     shadow=self.net.shadow)
            self.obs_bf16 = torch.zeros(N, 8, device=self.device, dtype=torch.bfloat16)
            self.mb_obs_bf16 = torch.zeros(cfg.minibatch_size, 8, device=self.device, dtype=torch.bfloat16)
            self.ws_roll = self.net.workspace(N)
            self.ws_mb = self.net.workspace(cfg.minibatch_size)
        else:
            self.policy = ActorCritic(4, 2, cfg.hidden, discrete=True, device=self.device, seed=cfg.seed)
            self.flat, self.flat_grad = self.policy.fp.flat, self.policy.fp.grad
            self.opt = FusedAdam(self.policy.fp.flat, self.policy.fp.grad, lr=cfg.lr,
                                 max_grad_norm=cfg.max_grad_norm)
        self.grad_sync = grad_sync
        self.state = self.env.state()  # live [N, 4] view
        self.ep_len, self.ep_ret, self.ep_count, self.ep_stats = self.env.episode_buffers()
        f32 = dict(device=self.device, dtype=torch.float32)
        self.obs_buf = torch.zeros(T, N, 4, **f32)
        self.act_buf = torch.zeros(T, N, device=self.device, dtype=torch.int32)
        self.logp_buf = torch.zeros(T, N, **f32)
        self.val_buf = torch.zeros(T + 1, N, **f32)
        self.rew_buf = torch.zeros(T, N, **f32)
        self.done_buf = torch.zeros(T, N, device=self.device, dtype=torch.uint8)
        self.adv = torch.zeros(T, N, **f32)
        self.ret = torch.zeros(T, N, **f32)
        self.adv_stats = torch.zeros(2, device=self.device, dtype=torch.float64)
        MB = cfg.minibatch_size
        self.mb_obs = torch.zeros(MB, 4, **f32)
        self.mb_act = torch.zeros(MB, device=self.device, dtype=torch.int32)
        self.mb_logp = torch.zeros(MB, **f32)
        self.mb_adv = torch.zeros(MB, **f32)
        self.mb_ret = torch.zeros(MB, **f32)
        self.loss_stats = torch.zeros(8, **f32)
        self.iter_t = torch.zeros(1, device=self.device, dtype=torch.int64)
        self.mb_step_t = torch.zeros(1, device=self.device, dtype=torch.int64)
        self.scratch = None
        self._empty_f32 = torch.empty(0, **f32)
        if self.cuda:
            n = _ops().gae_scratch_numel(T, N)
            self.scratch = torch.empty(max(n, 1), **f32)
        self.policy_seed = (cfg.seed * 0x9E3779B1 + rank * 0x85EBCA6B + 1) & 0xFFFFFFFFFFFF
        self.env_seed = self.env.seed()
        self._graphs = None
        self.iteration = 0
        self._cpu_gen = torch.Generator().manual_seed(cfg.seed + 1000 * rank)

    # ------------------------------------------------------------------ GPU
    def _autocast(self):
        if self.cuda and self.cfg.compute_dtype == "bf16":
            return torch.autocast("cuda", dtype=torch.bfloat16)
        return torch.autocast("cuda", enabled=False) if self.cuda else torch.autocast("cpu", enabled=False)

    def _rollout_gpu(self):
        o = _ops()
        T = self.cfg.rollout_steps
        params = {}
        if self.fused:
            o.pad_obs_bf16(self.state, self.obs_bf16)
            for t in range(T):
                logits, v = self.net.forward(self.obs_bf16, self.ws_roll)
                o.ppo_cartpole_act_step(logits, 2, v, self.state, self.obs_bf16, self.ep_len, self.ep_ret,
                                        self.ep_count, self.ep_stats, self.obs_buf, self.act_buf, self.logp_buf,
                                        self.val_buf, self.rew_buf, self.done_buf, self.iter_t, t, self.policy_seed,
                                        self.env_seed, params)
            _, v = self.net.forward(self.obs_bf16, self.ws_roll)
            self.val_buf[T].copy_(v[:, 0])
        else:
          with torch.no_grad(), self._autocast():
            for t in range(T):
                logits, v = self.policy(self.state)
                o.ppo_cartpole_act_step(logits.float().contiguous(), 2, v.float().contiguous(), self.state, None,
                                        self.ep_len, self.ep_ret, self.ep_count, self.ep_stats, self.obs_buf,
                                        self.act_buf, self.logp_buf, self.val_buf, self.rew_buf, self.done_buf,
                                        self.iter_t, t, self.policy_seed, self.env_seed, params)
            self.val_buf[T].copy_(self.policy.critic(self.state).float())
        self.adv_stats.zero_()
        gae(self.rew_buf, self.val_buf, self.done_buf, self.cfg.gamma, self.cfg.lam, stats=self.adv_stats,
            scratch=self.scratch, out=(self.adv, self.ret))
        self.mb_step_t.zero_()

    def _minibatch_gpu(self):
        self._minibatch_grad_gpu()
        self._minibatch_apply_gpu(self._sync_grads())

    def _sync_grads(self):
        return self.grad_sync(self.flat_grad) if self.grad_sync is not None else 1.0

    def _minibatch_apply_gpu(self, scale):
        if self.dp == "fused":
            self.opt.step()  # reduce-scatter + sharded Adam + all-gather (mean over ranks)
        else:
            self.opt.step(grad_scale=scale)
        _ops().counter_add(self.mb_step_t, 1)

    def _minibatch_grad_gpu(self):
        cfg = self.cfg
        o = _ops()
        if self.fused:
            o.ppo_gather(self.obs_buf, self.act_buf, self.logp_buf, self.adv, self.ret, self.val_buf, self.adv_stats,
                         self._empty_f32, self.mb_act, self.mb_logp, self.mb_adv, self.mb_ret, None,
                         cfg.n_minibatches, self.mb_step_t, self.iter_t, 0, self.policy_seed ^ 0x5851F42D,
                         cfg.norm_adv, self.mb_obs_bf16)
            if self.net.fused_head:  # output layer + loss + output-layer backward in one pass over H2
                self.net.forward_hidden(self.mb_obs_bf16, self.ws_mb)
                self.net.loss_backward(self.mb_obs_bf16, self.ws_mb, self.mb_act, self.mb_logp, self.mb_adv,
                                       self.mb_ret, self.loss_stats, cfg.clip, cfg.vf_coef, cfg.ent_coef)
                return
            logits, v = self.net.forward(self.mb_obs_bf16, self.ws_mb)
            o.ppo_loss_padded(logits, 2, v, self.mb_act, self.mb_logp, self.mb_adv, self.mb_ret, self.ws_mb["dlog"],
                              self.ws_mb["dval"], self.loss_stats, cfg.clip, cfg.vf_coef, cfg.ent_coef,
                              self.net.g["b3a"], self.net.g["b3c"])
            self.net.backward(self.mb_obs_bf16, self.ws_mb, out_bias_grads_done=True)
            return
        o.ppo_gather(self.obs_buf, self.act_buf, self.logp_buf, self.adv, self.ret, self.val_buf, self.adv_stats,
                     self.mb_obs, self.mb_act, self.mb_logp, self.mb_adv, self.mb_ret, None, cfg.n_minibatches,
                     self.mb_step_t, self.iter_t, 0, self.policy_seed ^ 0x5851F42D, cfg.norm_adv)
        self.policy.fp.grad.zero_()
        with self._autocast():
            logits, v = self.policy(self.mb_obs)
        loss = ppo_categorical_loss(logits.float(), v.float(), self.mb_act, self.mb_logp, self.mb_adv, self.mb_ret,
                                    cfg.clip, cfg.vf_coef, cfg.ent_coef, stats=self.loss_stats)
        loss.backward()

    def _end_iteration_gpu(self):
        _ops().counter_add(self.iter_t, 1)

    def _sync_capturable(self) -> bool:
        return self.grad_sync is None or getattr(self.grad_sync, "capturable", False)

    def check_collectives(self):
        """Raises if a peer-memory collective timed out (reads a device word)."""
        for obj in (self.opt, self.grad_sync):
            if hasattr(obj, "check"):
                obj.check()

    def _build_graphs(self):
        if not (self.cuda and self.cfg.cuda_graphs):
            return
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        # Warm-up on a side stream (autograd/cuBLAS workspaces get allocated
        # here, outside capture).  This advances the env and the optimizer
        # state once, which is harmless: it is one real training step.
        with torch.cuda.stream(s):
            self._rollout_gpu()
            for _ in range(2):
                self._minibatch_gpu()
            self._end_iteration_gpu()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        pool = torch.cuda.graph_pool_handle()
        g_roll, g_end = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_roll, pool=pool):
            self._rollout_gpu()
        if self._sync_capturable():
            g_mb = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_mb, pool=pool):
                self._minibatch_gpu()
            mb = (g_mb,)
        else:
            # a library collective stays outside the graphs: grads -> sync -> apply
            scale = getattr(self.grad_sync, "scale", 1.0)
            g_grad, g_apply = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_grad, pool=pool):
                self._minibatch_grad_gpu()
            with torch.cuda.graph(g_apply, pool=pool):
                self._minibatch_apply_gpu(scale)
            mb = (g_grad, g_apply)
        with torch.cuda.graph(g_end, pool=pool):
            self._end_iteration_gpu()
        torch.cuda.synchronize(self.device)
        if not self.fused:
            self.policy.fp.rebind_grads()
        self._graphs = (g_roll, mb, g_end)

    def release_graphs(self):
        self._graphs = None

    # ------------------------------------------------------------------ CPU
    def _rollout_cpu(self):
        T = self.cfg.rollout_steps
        if getattr(self, "host_rollout", True):
            # the T steps in one call into the core: policy forward, sampling
            # (Philox uniform of (policy seed; env, step, iteration), inverse
            # CDF), environment step and buffers; the loop below is the
            # torch-op path with the same buffer layout
            cfg = self.cfg
            _core().ppo_cartpole_rollout_host(self.env, self.policy.fp.flat.detach(), [4, *cfg.hidden, 2],
                                              [4, *cfg.hidden, 1], self.obs_buf, self.act_buf, self.logp_buf,
                                              self.val_buf, self.rew_buf, self.done_buf, self.policy_seed,
                                              self.iteration)
            gae(self.rew_buf, self.val_buf, self.done_buf, cfg.gamma, cfg.lam, out=(self.adv, self.ret))
            return
        with torch.no_grad():
            for t in range(T):
                logits, v = self.policy(self.state)
                logp_all = F.log_softmax(logits.float(), -1)
                g = -torch.log(-torch.log(torch.rand(logits.shape, generator=self._cpu_gen).clamp_(1e-9, 1 - 1e-7)))
                a = (logits + g).argmax(-1).to(torch.int32)
                self.obs_buf[t].copy_(self.state)
                self.act_buf[t].copy_(a)
                self.logp_buf[t].copy_(logp_all.gather(1, a.long()[:, None]).squeeze(1))
                self.val_buf[t].copy_(v)
                obs = torch.empty_like(self.state)
                rew = torch.empty(self.state.shape[0])
                done = torch.empty(self.state.shape[0], dtype=torch.bool)
                self.env.step_into(a, obs, rew, done)
                self.rew_buf[t].copy_(rew)
                self.done_buf[t].copy_(done.to(torch.uint8))
            self.val_buf[T].copy_(self.policy.critic(self.state))
        adv, ret = ref.gae(self.rew_buf, self.val_buf, self.done_buf, self.cfg.gamma, self.cfg.lam)
        self.adv.copy_(adv)
        self.ret.copy_(ret)

    def _update_cpu(self):
        cfg = self.cfg
        B = cfg.batch
        obs = self.obs_buf.view(B, 4)
        act, logp, adv, ret = (x.reshape(B) for x in (self.act_buf, self.logp_buf, self.adv, self.ret))
        if cfg.norm_adv:
            adv = (adv - adv.mean()) / (adv.std() + 1e-8)
        # the minibatch step in the core (forward, loss and hand-written
        # backward, no autograd graph), or through autograd when host_update
        # is off; both compute the same gradient
        host = getattr(self, "host_update", True)
        dims_a, dims_c = [4, *cfg.hidden, 2], [4, *cfg.hidden, 1]
        flat = self.policy.fp.flat.detach()
        adv = adv.contiguous()
        if host and self.grad_sync is None:
            # the whole update in one call: the same minibatch order (one
            # permutation per epoch from the trainer's generator) and Adam steps
            perms = torch.stack([torch.randperm(B, generator=self._cpu_gen) for _ in range(cfg.epochs)])
            o = self.opt
            o._host_step = int(_core().ppo_update_host(
                flat, self.flat_grad, o.m, o.v, o._host_step, dims_a, dims_c, obs, act, logp, adv, ret, perms,
                cfg.minibatch_size, cfg.clip, cfg.vf_coef, cfg.ent_coef, o.lr, o.betas[0], o.betas[1], o.eps, o.wd,
                self.loss_stats))
            return
        for _ in range(cfg.epochs):
            perm = torch.randperm(B, generator=self._cpu_gen)
            for k in range(cfg.n_minibatches):
                idx = perm[k * cfg.minibatch_size:(k + 1) * cfg.minibatch_size]
                self.policy.fp.grad.zero_()
                if host:
                    _core().ppo_minibatch_host(flat, self.flat_grad, dims_a, dims_c, obs, act, logp, adv, ret, idx,
                                               cfg.clip, cfg.vf_coef, cfg.ent_coef, self.loss_stats)
                else:
                    logits, v = self.policy(obs[idx])
                    loss = ppo_categorical_loss(logits, v, act[idx], logp[idx], adv[idx], ret[idx], cfg.clip,
                                                cfg.vf_coef, cfg.ent_coef, stats=self.loss_stats)
                    loss.backward()
                scale = self.grad_sync(self.flat_grad) if self.grad_sync is not None else 1.0
                self.opt.step(grad_scale=scale)

    # ------------------------------------------------------------------ API
    def train_iteration(self):
        """Runs one rollout + update.  Returns nothing (metrics are read
        lazily by :meth:`metrics`, which synchronizes)."""
        cfg = self.cfg
        if not self.cuda:
            prev = torch.get_num_threads()
            want = cfg.cpu_threads
            if want <= 0:
                host = getattr(self, "host_update", True) and getattr(self, "host_rollout", True)
                small = cfg.minibatch_size * max(cfg.hidden or (1,)) <= 65536
                want = prev if host or not small else 1
            if want != prev:
                torch.set_num_threads(want)
            try:
                self._rollout_cpu()
                self._update_cpu()
            finally:
                if want != prev:
                    torch.set_num_threads(prev)
            self.iteration += 1
            return
        if cfg.cuda_graphs and self._graphs is None:
            self._build_graphs()
        if self._graphs is not None:
            g_roll, mb, g_end = self._graphs
            g_roll.replay()
            if len(mb) == 1:
                for _ in range(cfg.epochs * cfg.n_minibatches):
                    mb[0].replay()
            else:
                for _ in range(cfg.epochs * cfg.n_minibatches):
                    mb[0].replay()
                    self.grad_sync(self.flat_grad)
                    mb[1].replay()
            g_end.replay()
        else:
            self._rollout_gpu()
            for _ in range(cfg.epochs * cfg.n_minibatches):
                self._minibatch_gpu()
            self._end_iteration_gpu()
        self.iteration += 1

    def metrics(self) -> dict:
        """Episode and loss statistics since the previous call (synchronizes)."""
        s = self.env.take_episode_stats()
        ls = self.loss_stats.double().cpu().tolist()
        self.loss_stats.zero_()
        n = max(ls[5], 1.0)
        out = {
            "episodes": s[1],
            "mean_return": s[0] / s[1] if s[1] > 0 else float("nan"),
            "mean_length": s[2] / s[1] if s[1] > 0 else float("nan"),
            "policy_loss": ls[0] / n,
            "value_loss": ls[1] / n,
            "entropy": ls[2] / n,
            "approx_kl": ls[3] / n,
            "clipfrac": ls[4] / n,
        }
        return out

    def env_steps_per_iteration(self) -> int:
        return self.cfg.batch

    def checkpoint_ranks(self) -> dict:
        """Place of this rank in a checkpoint: with data parallelism every rank
        saves its own environments, RNG and (fused step) optimizer shard; the
        policy is the same on every rank and is written by rank 0."""
        if self.dp == "none":
            return {}
        import torch.distributed as dist

        return {"dp_rank": dist.get_rank(self.group), "layout": {"tp": 1, "pp": 1, "dp": dist.get_world_size(self.group)}}

    def state_dict(self):
        pol = self.net.state_dict() if self.fused else self.policy.state_dict()
        return {"policy": pol, "optim": self.opt.state_dict(), "iteration": self.iteration,
                "iter_t": self.iter_t.clone(), "env_state": self.state.clone(),
                "ep": (self.ep_len.clone(), self.ep_ret.clone(), self.ep_count.clone()),
                "cpu_rng": self._cpu_gen.get_state()}

    def load_state_dict(self, sd):
        with torch.no_grad():
            if self.fused:
                self.net.load_state_dict(sd["policy"])
            else:
                self.policy.load_state_dict(sd["policy"])
            self.opt.load_state_dict(sd["optim"])
            self.iteration = int(sd["iteration"])
            self.iter_t.copy_(sd["iter_t"])
            self.state.copy_(sd["env_state"])
            for dst, src in zip((self.ep_len, self.ep_ret, self.ep_count), sd["ep"]):
                dst.copy_(src)
            if "cpu_rng" in sd:
                self._cpu_gen.set_state(sd["cpu_rng"])
