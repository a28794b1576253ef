"""GRPO (Shao et al. 2024, "DeepSeekMath", group relative policy optimization)
for a decoder-only policy on the turbol_b200 kernels.

One step:
  1. rollout   P prompts x G samples, ``response_len`` tokens each, temperature
               sampling (LLMGenerator: own paged-KV decode loop, CUDA graph);
  2. reward    R = (FNV-1a-64(response ids) mod 1000) / 1000 (hash reward
               kernel) -> group-normalized advantages (GRPO kernel);
  3. reference log-probs of the sampled responses under the frozen initial
               policy (forward only);
  4. update    micro-batched forward with saved activations -> LM-head logits
               of the response positions -> log-probs -> GRPO loss kernel
               (clipped ratio, k3 KL to the reference, per-sequence token mean)
               -> logits gradient in place -> hand-written backward -> fp32
               gradient accumulation -> one fused Adam launch over all weights.
With one update per rollout the behaviour policy equals the current policy,
so the ratio is 1 and the clip is inactive (the GRPO setting with mu = 1).

Train tokens per step = P * G * (prompt_len + response_len).

The reference's grpo_example.py (turbol_vllm/examples/py/grpo_example.py:124-151)
echoes prompts and updates a linear policy on an uninitialised batch; this
module is the algorithm it names.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from .._native import ops as _ops
from ..models.llm import DecoderLM, LMConfig
from ..ops.rl import FusedAdam
from .rollout import LLMGenerator


@dataclass
class GRPOConfig:
    model: LMConfig = field(default_factory=LMConfig.qwen2_1p5b)
    num_prompts: int = 64
    group_size: int = 8
    prompt_len: int = 256
    response_len: int = 512
    temperature: float = 1.0
    lr: float = 1e-6
    clip: float = 0.2
    kl_coef: float = 0.04
    micro_batch: int = 8  # sequences per forward/backward
    seed: int = 0

    @property
    def batch(self) -> int:
        return self.num_prompts * self.group_size

    @property
    def seq_len(self) -> int:
        return self.prompt_len + self.response_len


class GRPOTrainer:
    """GRPO on one GPU, or data-parallel over a process group.

    dp: "none"; "fused" (gradient reduce-scatter, sharded Adam and weight
    all-gather in one NVLink peer-memory kernel; the model's fp32 weights,
    gradient and bf16 copy live in symmetric memory); "nccl" (NCCL all-reduce
    of the gradient + local fused Adam; the baseline).  With data parallelism
    ``cfg.num_prompts`` is per rank and every rank samples its own prompts.

    tp > 1: groups of ``tp`` consecutive ranks generate ``cfg.num_prompts``
    prompts together with a tensor-parallel rollout (TPLLMGenerator on the
    fused all-gather->GEMM / GEMM->reduce-scatter kernels).  ``tp_mode``:

    * "train" (default): training is tensor parallel too (TPTrainLM: each rank
      owns 1/tp of every projection, forward and backward on the fused
      kernels); the TP group trains on all of its sequences, each micro-batch
      split by rows over the ranks; data parallelism (``dp``) runs over the
      ranks that hold the same shard (TP x DP).  The rollout and the frozen
      reference model are per-rank full copies by default (``rollout``
      below), so decoding and reference scoring need no collective.
    * "rollout": every rank keeps the full model and trains data parallel on
      its 1/tp share of the group's sequences; after the optimizer step every
      rank re-slices its rollout shard from the updated weights."""

    def __init__(self, cfg: GRPOConfig, device="cuda:0", optimizer=None, dp: str = "none", group=None,
                 tp: int = 1, tp_mode: str = "train", rollout: str = "replica"):
        """rollout (tp_mode "train"): "replica" - each rank decodes its share of
        the group's sequences on a full bf16 copy of the model that a fused
        all-gather kernel refreshes after every optimizer step
        (:class:`~turbol_b200.parallel.weight_sync.TPReplicaSync`); "tp" - the
        tensor-parallel decode on the trainer's own shards (no copy, two fused
        collectives per layer per token)."""
        self.cfg = cfg
        self.rollout_mode = rollout if tp > 1 and tp_mode == "train" else "local"
        if self.rollout_mode not in ("replica", "tp", "local"):
            raise ValueError(f"unknown rollout mode {rollout!r}")
        self.sync = None
        self.device = torch.device(device)
        self.dp, self.group = dp, group
        self.rank, self.world = 0, 1
        if dp != "none":
            import torch.distributed as dist

            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.tp, self.tp_mode = tp, tp_mode if tp > 1 else "none"
        self.tp_rank, self.group_index = 0, self.rank
        self.grad_sync = None
        if tp > 1 and tp_mode == "train":
            self._init_tp_train(cfg, dp)
            return
        if tp > 1 and tp_mode != "rollout":
            raise ValueError(f"unknown tensor-parallel mode {tp_mode!r}")
        self.model = DecoderLM(cfg.model, self.device, seed=cfg.seed)
        if dp == "fused":
            from ..parallel.peer import FusedDataParallelAdam

            self.opt = FusedDataParallelAdam(self.model.numel, group, lr=cfg.lr, betas=(0.9, 0.95))
            self.model.rebind_storage(self.opt.param, self.opt.grad, self.opt.shadow)
            self.opt.broadcast_params(0)
        else:
            self.opt = optimizer or FusedAdam(self.model.flat, self.model.grad, lr=cfg.lr, betas=(0.9, 0.95),
                                              shadow=self.model.shadow)
            if dp == "nccl":
                import torch.distributed as dist

                from ..parallel.dp import NcclGradSync

                dist.broadcast(self.model.flat, src=0, group=group)
                self.model.sync_shadow()
                self.grad_sync = NcclGradSync(group)
            elif dp != "none":
                raise ValueError(f"unknown data-parallel mode {dp!r}")
        self.ref = self.model.frozen_copy()
        if tp > 1:
            from ..models.tp_llm import TPDecoderLM
            from ..parallel.dist import build_mesh
            from ..parallel.tp import TensorParallelComm
            from .rollout import TPLLMGenerator

            if dp == "none":
                raise ValueError("tensor-parallel rollout needs a process group (dp='fused' or 'nccl')")
            mesh = build_mesh(self.world, self.rank, tp=tp)
            self.tp_rank, self.group_index = mesh.tp_rank, self.rank // tp
            rows = max(cfg.num_prompts * cfg.prompt_len, cfg.batch)
            self.comm = TensorParallelComm(rows, cfg.model.hidden, cfg.model.hidden, group=mesh.tp_group,
                                           device=self.device.index)
            self.tpm = TPDecoderLM(self.model, self.comm)
            self.gen = TPLLMGenerator(self.tpm, cfg.batch, cfg.seq_len, seed=cfg.seed + 17 + 7919 * self.group_index)
        else:
            self.gen = LLMGenerator(self.model, cfg.batch, cfg.seq_len, seed=cfg.seed + 17 + 7919 * self.rank)
        self.stats = torch.zeros(4, device=self.device)
        self.step_count = 0
        self.last_times = {}

    def _init_tp_train(self, cfg: GRPOConfig, dp: str):
        """TP x DP training: the model is this rank's shard (TPTrainLM)."""
        import torch.distributed as dist

        from ..models.tp_llm import TPTrainLM
        from ..parallel.dist import build_mesh
        from ..parallel.tp import TensorParallelComm
        from .rollout import TPLLMGenerator

        tp = self.tp
        if dp == "none":
            raise ValueError("tensor-parallel training needs a process group (dp='fused' or 'nccl')")
        if cfg.micro_batch % tp or (cfg.micro_batch // tp * cfg.seq_len) % 128 or cfg.batch % cfg.micro_batch:
            raise ValueError("tensor-parallel training: micro_batch must divide the batch, split over the TP ranks "
                             "into whole sequences, and give each rank a multiple of 128 rows")
        # the fused TP kernels work on 128-row tiles of each rank's share: prefill
        # rows (prompts x prompt_len) and decode rows (sequences) per rank
        if (cfg.num_prompts * cfg.prompt_len // tp) % 128 or (cfg.batch // tp) % 128 or cfg.num_prompts % tp:
            raise ValueError("tensor-parallel rollout: each rank needs a multiple of 128 prompt tokens and of 128 "
                             f"sequences (num_prompts={cfg.num_prompts}, prompt_len={cfg.prompt_len}, "
                             f"batch={cfg.batch}, tp={tp})")
        mesh = build_mesh(self.world, self.rank, tp=tp)
        self.mesh = mesh
        self.tp_rank, self.group_index = mesh.tp_rank, self.rank // tp
        H = cfg.model.hidden
        rows = max(cfg.num_prompts * cfg.prompt_len, cfg.batch, cfg.micro_batch * cfg.seq_len)
        self.comm = TensorParallelComm(rows, H, H, group=mesh.tp_group, device=self.device.index)
        full = DecoderLM(cfg.model, self.device, seed=cfg.seed, master=False)  # bf16 only, sliced below
        self.model = TPTrainLM(full, self.comm)
        dp_world = mesh.dp
        if dp_world > 1 and dp == "fused":
            from ..parallel.peer import FusedDataParallelAdam

            self.opt = FusedDataParallelAdam(self.model.numel, mesh.dp_group, lr=cfg.lr, betas=(0.9, 0.95))
            self.model.rebind_storage(self.opt.param, self.opt.grad, self.opt.shadow)
            self.opt.broadcast_params(0)
        else:
            self.opt = FusedAdam(self.model.flat, self.model.grad, lr=cfg.lr, betas=(0.9, 0.95),
                                 shadow=self.model.shadow)
            if dp_world > 1:
                from ..parallel.dp import NcclGradSync

                dist.broadcast(self.model.flat, src=dist.get_global_rank(mesh.dp_group, 0), group=mesh.dp_group)
                self.model.shadow.copy_(self.model.flat)
                self.grad_sync = NcclGradSync(mesh.dp_group)
        if self.rollout_mode == "replica":
            # the frozen reference stays a whole bf16 model (the initial
            # weights): each rank scores its own sequences with it, no collective
            self.ref = full
        else:
            self.ref = self.model.frozen_copy()
        del full
        self.tpm = self.model
        if self.rollout_mode == "replica":
            from ..parallel.weight_sync import TPReplicaSync

            self.sync = TPReplicaSync(self.model, mesh.tp_group)
            self.sync()
            self.gen = LLMGenerator(self.sync.full, cfg.batch // tp, cfg.seq_len,
                                    seed=cfg.seed + 17 + 7919 * self.group_index + 104729 * self.tp_rank)
        else:
            self.gen = TPLLMGenerator(self.model, cfg.batch, cfg.seq_len,
                                      seed=cfg.seed + 17 + 7919 * self.group_index)
        self.stats = torch.zeros(4, device=self.device)
        self.step_count = 0
        self.last_times = {}

    # ------------------------------------------------------------------ checkpoint
    def checkpoint_ranks(self) -> dict:
        """Place of this rank in a checkpoint.  Tensor-parallel training: one
        policy file per TP shard (``_tp<t>_pp0``), optimizer and trainer state
        per data-parallel rank of that shard.  Full-model data parallelism: one
        policy file, optimizer/trainer state per rank."""
        if self.tp_mode == "train":
            return {"tp_rank": self.tp_rank, "pp_rank": 0, "dp_rank": self.mesh.dp_rank,
                    "layout": {"tp": self.tp, "pp": 1, "dp": self.mesh.dp}}
        if self.dp != "none":
            return {"dp_rank": self.rank, "layout": {"tp": 1, "pp": 1, "dp": self.world}}
        return {}

    def state_dict(self) -> dict:
        """Master weights (fp32), the frozen reference weights, optimizer state and
        the step counter (which also keys the prompt and sampling streams)."""
        return {"policy": {"flat": self.model.flat, "shadow": self.model.shadow},
                "optim": self.opt.state_dict(), "ref_shadow": self.ref.shadow,
                "step_count": self.step_count, "gen_calls": self.gen.calls}

    def load_state_dict(self, sd: dict):
        with torch.no_grad():
            self.model.flat.copy_(sd["policy"]["flat"])
            self.model.shadow.copy_(sd["policy"]["shadow"])
            self.ref.shadow.copy_(sd["ref_shadow"])
            self.ref._make_views()  # a bf16-only model keeps fp32 copies of its norms and biases: refresh them
            self.opt.load_state_dict(sd["optim"])
            if self.tp_mode == "rollout":
                self.tpm.load_from(self.model)  # the rollout shard follows the loaded weights
            elif self.sync is not None:
                self.sync()  # and the rollout replicas
        self.step_count = int(sd["step_count"])
        self.gen.calls = int(sd["gen_calls"])

    # ------------------------------------------------------------------ helpers
    def _replica_rollout(self):
        """Rank r of the TP group decodes prompts [r P/tp, (r+1) P/tp) (x G
        samples) on its replica; the group then shares all sequences (in
        prompt order) for the tensor-parallel update."""
        import torch.distributed as dist

        cfg, tp, r = self.cfg, self.tp, self.tp_rank
        P = cfg.num_prompts // tp
        prompts = self._prompts()[r * P:(r + 1) * P].contiguous()
        seqs, lp = self.gen.generate(prompts, cfg.group_size, cfg.response_len, cfg.temperature)
        g = self.mesh.tp_group
        all_seqs = torch.empty((tp,) + tuple(seqs.shape), device=self.device, dtype=seqs.dtype)
        all_lp = torch.empty((tp,) + tuple(lp.shape), device=self.device, dtype=lp.dtype)
        dist.all_gather_into_tensor(all_seqs, seqs.contiguous(), group=g)
        dist.all_gather_into_tensor(all_lp, lp.contiguous(), group=g)
        return all_seqs.view(-1, seqs.shape[1]), all_lp.view(-1, lp.shape[1])

    def _prompts(self) -> torch.Tensor:
        g = torch.Generator(device=self.device).manual_seed(self.cfg.seed * 1000003 + self.step_count +
                                                            104729 * self.group_index)
        return torch.randint(0, self.cfg.model.vocab, (self.cfg.num_prompts, self.cfg.prompt_len),
                             generator=g, device=self.device, dtype=torch.int32)

    def _response_rows(self, m: int) -> torch.Tensor:
        """Indices of the hidden rows that predict the response tokens of m sequences."""
        T, Lp, Lr = self.cfg.seq_len, self.cfg.prompt_len, self.cfg.response_len
        base = torch.arange(m, device=self.device) * T
        return (base[:, None] + torch.arange(Lp - 1, Lp - 1 + Lr, device=self.device)[None, :]).reshape(-1)

    @torch.no_grad()
    def ref_logprobs(self, seqs: torch.Tensor) -> torch.Tensor:
        """Log-probs of the response tokens under the frozen reference model."""
        cfg = self.cfg
        o = _ops()
        B, T, Lr = seqs.shape[0], cfg.seq_len, cfg.response_len
        out = torch.empty(B, Lr, device=self.device)
        mb = cfg.micro_batch
        pos = torch.arange(T, device=self.device, dtype=torch.int32).repeat(mb)
        for s0 in range(0, B, mb):
            ids = seqs[s0:s0 + mb].contiguous()
            m = ids.shape[0]
            x = self.ref.embed(ids)
            x, _ = self.ref.forward(x, m, T, pos[: m * T], save=False)
            hf = self.ref.final_norm(x)
            rows = hf.index_select(0, self._response_rows(m))
            logits = self.ref.logits(rows)
            tgt = ids[:, cfg.prompt_len:].reshape(-1).contiguous()
            o.logprob(logits, tgt, out[s0:s0 + m].view(-1))
        return out

    # ------------------------------------------------------------------ step
    def step(self) -> dict:
        cfg = self.cfg
        o = _ops()
        dev = self.device
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        # 1. rollout
        if self.rollout_mode == "replica":
            seqs, roll_lp = self._replica_rollout()
        else:
            seqs, roll_lp = self.gen.generate(self._prompts(), cfg.group_size, cfg.response_len, cfg.temperature)
        torch.cuda.synchronize(dev)
        t1 = time.perf_counter()
        # 2. rewards and group-normalized advantages
        resp = seqs[:, cfg.prompt_len:].contiguous()
        lens = torch.full((cfg.batch,), cfg.response_len, device=dev, dtype=torch.int32)
        rewards = o.hash_reward(resp, lens)
        adv = o.grpo_advantage(rewards, cfg.group_size, 1e-4, True)
        if self.tp_mode == "rollout":  # this rank trains on its share of the tensor-parallel group's sequences
            share = cfg.batch // self.tp
            lo = self.tp_rank * share
            seqs, adv = seqs[lo:lo + share].contiguous(), adv[lo:lo + share].contiguous()
        train_tokens = seqs.shape[0] * cfg.seq_len // (self.tp if self.tp_mode == "train" else 1)
        # 3. reference log-probs
        if self.tp_mode == "train":
            own = self._tp_own(seqs.shape[0])
            adv = adv.index_select(0, own).contiguous()
            ref_lp = (self.ref_logprobs(seqs.index_select(0, own).contiguous()) if self.rollout_mode == "replica"
                      else self._tp_ref_logprobs(seqs))
        else:
            ref_lp = self.ref_logprobs(seqs)
        torch.cuda.synchronize(dev)
        t2 = time.perf_counter()
        # 4. update
        self.model.zero_grad()
        self.stats.zero_()
        if self.tp_mode == "train":
            self._train_tp(seqs, ref_lp, adv)
            self.model.reduce_replicated_grads()
            import torch.distributed as dist

            dist.all_reduce(self.stats, group=self.mesh.tp_group)
        else:
            self._train(seqs, ref_lp, adv)
        if self.grad_sync is not None:
            self.opt.step(grad_scale=self.grad_sync(self.model.grad))
        else:
            self.opt.step()  # the fused data-parallel step averages over ranks itself
        if self.tp_mode == "rollout":
            self.tpm.load_from(self.model)  # trainer -> rollout weight sync
        elif self.sync is not None:
            self.sync()  # fused all-gather of the new shards into every rank's rollout replica
        # (rollout "tp": the rollout reads the weights the optimizer just wrote)
        torch.cuda.synchronize(dev)
        t3 = time.perf_counter()
        self.step_count += 1
        st = self.stats.cpu().tolist()
        self.last_times = {"rollout_s": t1 - t0, "reward_ref_s": t2 - t1, "train_s": t3 - t2, "step_s": t3 - t0}
        return {"reward_mean": float(rewards.mean()), "reward_std": float(rewards.std()),
                "pg_loss": st[0], "kl": st[1], "clipped_tokens": st[2], "tokens": st[3],
                "rollout_logp_mean": float(roll_lp.mean()), **self.last_times,
                "train_tokens": train_tokens}

    def _train(self, seqs, ref_lp, adv):
        cfg = self.cfg
        o = _ops()
        m_ = self.model
        T, Lp, Lr = cfg.seq_len, cfg.prompt_len, cfg.response_len
        mb = cfg.micro_batch
        H = cfg.model.hidden
        pos = torch.arange(T, device=self.device, dtype=torch.int32).repeat(mb)
        mask = torch.ones(mb, Lr, device=self.device)
        nb = seqs.shape[0]
        for s0 in range(0, nb, mb):
            ids = seqs[s0:s0 + mb].contiguous()
            m = ids.shape[0]
            N = m * T
            x0 = m_.embed(ids)
            x, saved = m_.forward(x0, m, T, pos[:N], save=True)
            rstd = torch.empty(N, device=self.device)
            hf = m_.final_norm(x, rstd)
            rows = self._response_rows(m)
            hr = hf.index_select(0, rows)
            logits = m_.logits(hr)                                      # [m*Lr, V] bf16
            tgt = ids[:, Lp:].reshape(-1).contiguous()
            lp = torch.empty(m * Lr, device=self.device)
            o.logprob(logits, tgt, lp)
            old = lp.detach().clone()                                   # behaviour policy == current
            dlp = torch.empty_like(lp)
            o.grpo_loss(lp.view(m, Lr), old.view(m, Lr), ref_lp[s0:s0 + m].contiguous(), adv[s0:s0 + m].contiguous(),
                        mask[:m], dlp.view(m, Lr), self.stats, cfg.clip, cfg.kl_coef, 1.0 / nb)
            o.logprob(logits, tgt, None, dlp)                          # logits <- d loss / d logits
            dhr = torch.empty(m * Lr, H, device=self.device, dtype=torch.bfloat16)
            o.gemm(logits, m_.head_weight(), dhr, False, True)          # d h = dLogits W_head
            o.gemm(logits, hr, m_.head_grad(), True, True, accumulate=True, split_k=1)  # dW_head += dLogits^T h
            dhf = torch.zeros(N, H, device=self.device, dtype=torch.bfloat16)
            dhf.index_copy_(0, rows, dhr)
            dx = torch.empty_like(x)
            o.rmsnorm_bwd(dhf, x, m_.f32["norm"], rstd, dx, None, m_.g["norm"])
            dx = m_.backward(dx, saved, m, T, pos[:N])
            m_.embed_backward(ids, dx)
            del saved, logits

    # ------------------------------------------------------------------ tensor-parallel training
    def _tp_own(self, nb: int) -> torch.Tensor:
        """Indices of the sequences whose rows this rank holds: in every
        micro-batch of ``micro_batch`` sequences, rank r holds the r-th 1/tp."""
        mb, tp, r = self.cfg.micro_batch, self.tp, self.tp_rank
        ml = mb // tp
        base = torch.arange(0, nb, mb, device=self.device)
        return (base[:, None] + r * ml + torch.arange(ml, device=self.device)[None, :]).reshape(-1)

    @torch.no_grad()
    def _tp_ref_logprobs(self, seqs: torch.Tensor) -> torch.Tensor:
        """Reference log-probs of this rank's sequences (TP forward of the frozen shard)."""
        cfg = self.cfg
        o = _ops()
        ref = self.ref
        B, T, Lp, Lr = seqs.shape[0], cfg.seq_len, cfg.prompt_len, cfg.response_len
        mb, tp, r = cfg.micro_batch, self.tp, self.tp_rank
        ml = mb // tp
        out = torch.empty(B // tp, Lr, device=self.device)
        pos = torch.arange(T, device=self.device, dtype=torch.int32).repeat(mb)
        rows = self._response_rows(ml)
        for j, s0 in enumerate(range(0, B, mb)):
            ids = seqs[s0:s0 + mb].contiguous()
            x = ref.embed_rows(ids.reshape(-1))
            x = ref.forward(x, mb, T, pos)
            hf = ref.final_norm(x)
            logits = ref.logits(hf.index_select(0, rows))
            tgt = ids[r * ml:(r + 1) * ml, Lp:].reshape(-1).contiguous()
            o.logprob(logits, tgt, out[j * ml:(j + 1) * ml].view(-1))
        return out

    def _train_tp(self, seqs, ref_lp, adv):
        """Micro-batched TP forward/backward; every rank of the group runs the
        same micro-batches, each on its rows (whole sequences)."""
        cfg = self.cfg
        o = _ops()
        M = self.model
        T, Lp, Lr = cfg.seq_len, cfg.prompt_len, cfg.response_len
        mb, tp, r = cfg.micro_batch, self.tp, self.tp_rank
        ml = mb // tp
        H = cfg.model.hidden
        nb = seqs.shape[0]
        pos = torch.arange(T, device=self.device, dtype=torch.int32).repeat(mb)
        mask = torch.ones(ml, Lr, device=self.device)
        rows = self._response_rows(ml)
        for j, s0 in enumerate(range(0, nb, mb)):
            ids = seqs[s0:s0 + mb].contiguous()
            x0 = M.embed_rows(ids.reshape(-1))
            x, saved = M.forward_train(x0, mb, T, pos, save=True)
            rstd = torch.empty(ml * T, device=self.device)
            hf = M.full.final_norm(x, rstd)
            hr = hf.index_select(0, rows)
            logits = M.full.logits(hr)                                  # [ml*Lr, V] bf16
            tgt = ids[r * ml:(r + 1) * ml, Lp:].reshape(-1).contiguous()
            lp = torch.empty(ml * Lr, device=self.device)
            o.logprob(logits, tgt, lp)
            old = lp.detach().clone()                                   # behaviour policy == current
            dlp = torch.empty_like(lp)
            sl = slice(j * ml, (j + 1) * ml)
            o.grpo_loss(lp.view(ml, Lr), old.view(ml, Lr), ref_lp[sl].contiguous(), adv[sl].contiguous(), mask,
                        dlp.view(ml, Lr), self.stats, cfg.clip, cfg.kl_coef, 1.0 / nb)
            o.logprob(logits, tgt, None, dlp)                          # logits <- d loss / d logits
            dhr = torch.empty(ml * Lr, H, device=self.device, dtype=torch.bfloat16)
            o.gemm(logits, M.full.head_weight(), dhr, False, True)      # d h = dLogits W_head
            o.gemm(logits, hr, M.full.head_grad(), True, True, accumulate=True, split_k=1)
            dhf = torch.zeros(ml * T, H, device=self.device, dtype=torch.bfloat16)
            dhf.index_copy_(0, rows, dhr)
            dx = torch.empty_like(x)
            o.rmsnorm_bwd(dhf, x, M.f32["norm"], rstd, dx, None, M.g["norm"])
            dx = M.backward(dx, saved, mb, T, pos)
            M.embed_backward_rows(ids.reshape(-1), dx)
            del saved, logits
