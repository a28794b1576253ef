"""PPO-RLHF on a pipeline-parallel decoder policy with a value head.

One step (every rank is one pipeline stage of the trainer and also holds a
bf16 rollout copy of the whole policy):

  1. weight sync   each stage broadcasts its bf16 weights into every rank's
                   rollout copy (NCCL broadcast per tensor);
  2. rollout       each rank samples responses for its share of the prompts
                   with its own paged-KV decode loop; the sequences are
                   all-gathered;
  3. scoring       a forward-only pipeline pass of the policy gives the
                   behaviour log-probs and values of the response tokens; one
                   of the frozen reference policy gives reference log-probs;
                   the last stage forms per-token rewards (KL penalty
                   -beta * (logp - logp_ref), plus the sequence reward
                   (hash(response) mod 1000) / 1000 on the last token) and
                   GAE(gamma, lambda) advantages (the GAE kernel), whitened;
  4. update        one 1F1B pipeline pass (NCCL send/recv between stages)
                   with the clipped PPO policy loss and the clipped value loss
                   on the last stage; Adam on every stage.

The reference has no RLHF trainer or pipeline execution
(turbol_vllm/src/distributed/pipeline_trainer.cpp:67-113 is a serial stub).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from .._native import ops as _ops
from ..models.llm import DecoderLM, LMConfig
from ..ops.rl import gae
from ..parallel import pipeline as pp
from .rollout import LLMGenerator


@dataclass
class RLHFConfig:
    model: LMConfig = field(default_factory=LMConfig.llama3_8b)
    num_prompts: int = 32       # sequences per step (the whole pipeline)
    prompt_len: int = 512
    response_len: int = 1024
    micro_batch: int = 4        # sequences per pipeline micro-batch
    lr: float = 1e-6
    clip: float = 0.2
    vclip: float = 0.2
    vf_coef: float = 0.1
    kl_coef: float = 0.05
    gamma: float = 1.0
    lam: float = 0.95
    temperature: float = 1.0
    seed: int = 0
    recompute: bool = False     # activation recomputation in the pipeline stages

    @property
    def seq_len(self) -> int:
        return self.prompt_len + self.response_len


class _Frozen:
    """Forward-only stand-in for a pipeline stage (the reference policy)."""

    def __init__(self, stage: pp.PipelineStage):
        self.model = stage.model.frozen_copy()
        self.cfg, self.device = stage.cfg, stage.device
        self.stage, self.num_stages = stage.stage, stage.num_stages
        self.first, self.last = stage.first, stage.last
        self.tp = getattr(stage, "tp", 1)


class PPORLHFTrainer:
    """tp > 1: the world is split into ``world / tp`` pipeline stages of ``tp``
    consecutive ranks; each stage's layers are tensor parallel (TPTrainLM on
    the fused all-gather->GEMM / GEMM->reduce-scatter kernels, forward and
    backward), every micro-batch's rows are split over the stage's TP ranks,
    and rank t of a stage exchanges its rows with rank t of the neighbouring
    stages (PP x TP)."""

    def __init__(self, cfg: RLHFConfig, device, group=None, tp: int = 1):
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.ranks = list(range(self.world)) if group is None else dist.get_process_group_ranks(group)
        if cfg.num_prompts % cfg.micro_batch or cfg.num_prompts % self.world:
            raise ValueError("num_prompts must divide by micro_batch and by the world size")
        self.tp, self.tp_rank = tp, 0
        comm = None
        if tp > 1:
            from ..parallel.dist import build_mesh
            from ..parallel.tp import TensorParallelComm

            if group is not None:
                raise ValueError("pipeline x tensor parallel runs on the world group")
            if self.world % tp or cfg.micro_batch % tp or (cfg.micro_batch // tp * cfg.seq_len) % 128:
                raise ValueError("tp must divide the world size and the micro-batch, with a multiple of 128 rows "
                                 "per rank")
            mesh = build_mesh(self.world, self.rank, tp=tp, pp=self.world // tp)
            self.mesh, self.tp_rank = mesh, mesh.tp_rank
            self.pp_ranks, self.pp_group, self.tp_group = mesh.pp_ranks, mesh.pp_group, mesh.tp_group
            stage_idx, n_stages = mesh.pp_rank, mesh.pp
            H = cfg.model.hidden
            comm = TensorParallelComm(cfg.micro_batch * cfg.seq_len, H, H, group=mesh.tp_group,
                                      device=self.device.index)
            self.tp_comm = comm
        else:
            self.pp_ranks, self.pp_group, self.tp_group = self.ranks, group, None
            stage_idx, n_stages = self.rank, self.world
        self.n_stages = n_stages
        self.stage = pp.PipelineStage(cfg.model, stage_idx, n_stages, self.device, seed=cfg.seed, value_head=True,
                                      lr=cfg.lr, tp_comm=comm, recompute=cfg.recompute)
        # a tied embedding lives on the first and the last stage: same initial
        # weights, and the two gradients are summed after every backward pass
        # (one group per TP rank: the first- and last-stage ranks holding it)
        self.tied = cfg.model.tie_embeddings and n_stages > 1
        self.embed_group = None
        if self.tied:
            for t in range(tp):
                ends = [self.ranks[t], self.ranks[(n_stages - 1) * tp + t]]
                g = dist.new_group(ends)
                if self.rank in ends:
                    self.embed_group = g
        if self.tied and (self.stage.first or self.stage.last):
            dist.broadcast(self.stage.model.p["embed"], src=self.pp_ranks[0], group=self.embed_group)
            self.stage.model.sync_shadow()
        self.ref = _Frozen(self.stage)
        # bf16 rollout copy of the whole policy on every rank
        self.rollout = DecoderLM(cfg.model, self.device, seed=cfg.seed, master=False)
        self.gen = LLMGenerator(self.rollout, cfg.num_prompts // self.world, cfg.seq_len,
                                seed=cfg.seed + 31 + 7919 * self.rank)
        self.step_count = 0
        self.sync_weights()

    # ------------------------------------------------------------ checkpoint
    def checkpoint_ranks(self) -> dict:
        """One shard per (tensor rank, pipeline stage): ``policy_tp<t>_pp<p>``."""
        return {"tp_rank": self.tp_rank, "pp_rank": self.stage.stage,
                "layout": {"tp": self.tp, "pp": self.n_stages, "dp": 0}}

    def state_dict(self) -> dict:
        """This rank's stage: fp32 master weights (+ value head), the frozen
        reference shard, optimizer state and the step counter (which keys the
        prompt and sampling streams)."""
        st = self.stage
        pol = {"flat": st.model.flat, "shadow": st.model.shadow}
        opt = {"stage": st.opt.state_dict()}
        if st.value_head:
            pol["value_head"] = st.vh
            opt["value_head"] = st.vh_opt.state_dict()
        return {"policy": pol, "optim": opt, "ref_shadow": self.ref.model.shadow, "step_count": self.step_count,
                "gen_calls": self.gen.calls}

    @torch.no_grad()
    def load_state_dict(self, sd: dict):
        st = self.stage
        st.model.flat.copy_(sd["policy"]["flat"])
        st.model.shadow.copy_(sd["policy"]["shadow"])
        st.opt.load_state_dict(sd["optim"]["stage"])
        if st.value_head:
            st.vh.copy_(sd["policy"]["value_head"])
            st.vh_opt.load_state_dict(sd["optim"]["value_head"])
            st.sync_value_head()
        self.ref.model.shadow.copy_(sd["ref_shadow"])
        self.ref.model._make_views()
        self.step_count = int(sd["step_count"])
        self.gen.calls = int(sd["gen_calls"])
        self.sync_weights()  # the rollout copy follows the loaded weights

    # ------------------------------------------------------------ weight sync
    @torch.no_grad()
    def sync_weights(self):
        """Every stage's bf16 weights -> every rank's rollout copy."""
        if self.tp > 1:
            return self._sync_weights_tp()
        for src in range(self.world):
            for name in self._stage_names(src):
                t = self.rollout.s[name]
                if src == self.rank:
                    t.copy_(self.stage.model.s[name])
                dist.broadcast(t, src=self.ranks[src], group=self.group)
        # fp32 norm weights / biases in place: the captured decode graph keeps their addresses
        for n, t in self.rollout.f32.items():
            t.copy_(self.rollout.s[n].float())

    @torch.no_grad()
    def _sync_weights_tp(self):
        """PP x TP: every rank's bf16 shard buffer is broadcast once (the
        replicated tensors only from TP rank 0) and written into the matching
        slices of every rank's full rollout copy."""
        from ..models.tp_llm import TPTrainLM

        cfg, tp = self.cfg.model, self.tp
        if not hasattr(self, "_sync_buf"):
            most = max(TPTrainLM.layout(cfg, pp.stage_layers(cfg.n_layers, self.n_stages, s), s == 0,
                                        s == self.n_stages - 1, tp)[2] for s in range(self.n_stages))
            self._sync_buf = torch.empty(most, device=self.device, dtype=torch.bfloat16)
        for src in range(self.world):
            s, t = src // tp, src % tp
            offs, rep, numel = TPTrainLM.layout(cfg, pp.stage_layers(cfg.n_layers, self.n_stages, s), s == 0,
                                                s == self.n_stages - 1, tp)
            buf = self.stage.model.shadow if src == self.rank else self._sync_buf[:numel]
            lo = 0 if t == 0 else rep
            dist.broadcast(buf[lo:numel], src=self.ranks[src], group=self.group)
            TPTrainLM.unshard_into(self.rollout, buf, offs, tp, t, shards_only=t > 0)

    def _stage_names(self, s: int):
        cfg = self.cfg.model
        names = []
        if s == 0:
            names.append("embed")
        for i in pp.stage_layers(cfg.n_layers, self.world, s):
            names += [n for n in self.rollout.offsets if n.startswith(f"l{i}.")]
        if s == self.world - 1:
            names.append("norm")
            if not cfg.tie_embeddings:
                names.append("lm_head")
        return names

    # ------------------------------------------------------------ helpers
    def _resp_rows(self, m: int) -> torch.Tensor:
        T, Lp, Lr = self.cfg.seq_len, self.cfg.prompt_len, self.cfg.response_len
        base = torch.arange(m, device=self.device) * T
        return (base[:, None] + torch.arange(Lp - 1, Lp - 1 + Lr, device=self.device)[None, :]).reshape(-1)

    def _head(self, model: DecoderLM, x_out: torch.Tensor, m: int, ids: torch.Tensor):
        """Final norm, response-row logits and log-probs of the target tokens."""
        o = _ops()
        N = x_out.shape[0]
        rstd = torch.empty(N, device=self.device)
        hf = model.final_norm(x_out, rstd)
        rows = self._resp_rows(m)
        hr = hf.index_select(0, rows)
        logits = model.logits(hr)
        tgt = ids[:, self.cfg.prompt_len:].reshape(-1).contiguous()
        lp = torch.empty(m * self.cfg.response_len, device=self.device)
        o.logprob(logits, tgt, lp)
        return hf, rstd, rows, hr, logits, tgt, lp

    def _pass(self, stage, seqs: torch.Tensor, train: bool, on_last):
        cfg = self.cfg
        mb, T = cfg.micro_batch, cfg.seq_len
        M = seqs.shape[0] // mb
        pos = torch.arange(T, device=self.device, dtype=torch.int32).repeat(mb)
        pp.set_micro_geometry(mb, T, pos)

        if self.tp > 1:
            def first(i):
                return stage.model.embed_rows(seqs[i * mb:(i + 1) * mb].reshape(-1))

            def back_first(i, dx):
                stage.model.embed_backward_rows(seqs[i * mb:(i + 1) * mb].reshape(-1), dx)
        else:
            def first(i):
                return stage.model.embed(seqs[i * mb:(i + 1) * mb])

            def back_first(i, dx):
                stage.model.embed_backward(seqs[i * mb:(i + 1) * mb], dx)

        pp.run_1f1b(stage, self.pp_ranks, M, mb * T // self.tp, first, on_last, back_first, group=self.pp_group,
                    forward_only=not train)

    def _own(self, i: int) -> slice:
        """The sequences of micro-batch i whose rows this rank holds (all of
        them without TP; the tp_rank-th 1/tp with it)."""
        mb = self.cfg.micro_batch
        ml = mb // self.tp
        return slice(i * mb + self.tp_rank * ml, i * mb + (self.tp_rank + 1) * ml)

    # ------------------------------------------------------------ step
    def step(self) -> dict:
        cfg = self.cfg
        o = _ops()
        dev = self.device
        B, Lr = cfg.num_prompts, cfg.response_len
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        # 1. weight sync (after the previous update)
        if self.step_count > 0:
            self.sync_weights()
        torch.cuda.synchronize(dev)
        t_sync = time.perf_counter()
        # 2. rollout
        g = torch.Generator(device=dev).manual_seed(cfg.seed * 1000003 + self.step_count * 131 + self.rank)
        prompts = torch.randint(0, cfg.model.vocab, (B // self.world, cfg.prompt_len), generator=g, device=dev,
                                dtype=torch.int32)
        seqs_local, _ = self.gen.generate(prompts, 1, Lr, cfg.temperature)
        seqs = torch.empty(B, cfg.seq_len, device=dev, dtype=torch.int32)
        dist.all_gather_into_tensor(seqs, seqs_local.contiguous(), group=self.group)
        torch.cuda.synchronize(dev)
        t_roll = time.perf_counter()
        # 3. behaviour log-probs / values, reference log-probs, rewards, advantages
        mb = cfg.micro_batch
        old_lp = torch.zeros(B, Lr, device=dev)
        old_v = torch.zeros(B, Lr, device=dev)
        ref_lp = torch.zeros(B, Lr, device=dev)
        st = self.stage

        ml = mb // self.tp

        def score_policy(i, x_out):
            sl = self._own(i)
            hf, _, rows, hr, logits, tgt, lp = self._head(st.model, x_out, ml, seqs[sl])
            old_lp[sl] = lp.view(ml, Lr)
            old_v[sl] = st.values(hr).view(ml, Lr)

        def score_ref(i, x_out):
            sl = self._own(i)
            *_, lp = self._head(self.ref.model, x_out, ml, seqs[sl])
            ref_lp[sl] = lp.view(ml, Lr)

        with torch.no_grad():
            self._pass(st, seqs, False, score_policy)
            self._pass(self.ref, seqs, False, score_ref)
            if self.tp > 1 and st.last:  # every TP rank of the last stage scored its own sequences
                for t_ in (old_lp, old_v, ref_lp):
                    dist.all_reduce(t_, group=self.tp_group)
        adv = ret = None
        seq_reward = None
        if st.last:
            resp = seqs[:, cfg.prompt_len:].contiguous()
            seq_reward = o.hash_reward(resp, torch.full((B,), Lr, device=dev, dtype=torch.int32))
            r = -cfg.kl_coef * (old_lp - ref_lp)
            r[:, -1] += seq_reward
            vals = torch.cat([old_v.t(), torch.zeros(1, B, device=dev)], 0).contiguous()  # [Lr + 1, B]
            a_t, ret_t = gae(r.t().contiguous(), vals, torch.zeros(Lr, B, device=dev, dtype=torch.uint8),
                             cfg.gamma, cfg.lam)
            adv, ret = a_t.t().contiguous(), ret_t.t().contiguous()
            adv = (adv - adv.mean()) / (adv.std() + 1e-8)
        torch.cuda.synchronize(dev)
        t_score = time.perf_counter()
        # 4. PPO update through the pipeline (1F1B)
        st.zero_grad()
        stats = torch.zeros(4, device=dev)
        norm = 1.0 / (B * Lr)

        def loss_last(i, x_out):
            sl = self._own(i)
            ids = seqs[sl]
            hf, rstd, rows, hr, logits, tgt, lp = self._head(st.model, x_out, ml, ids)
            v = st.values(hr).contiguous()
            # clipped policy loss + clipped value loss, forward and backward in one kernel
            dlp, dv = torch.empty_like(lp), torch.empty_like(v)
            o.ppo_token_loss(lp, old_lp[sl].reshape(-1), adv[sl].reshape(-1), v, old_v[sl].reshape(-1),
                             ret[sl].reshape(-1), dlp, dv, stats, cfg.clip, cfg.vclip, cfg.vf_coef, norm)
            H = cfg.model.hidden
            o.logprob(logits, tgt, None, dlp)                                     # logits <- d loss / d logits
            dhr = torch.empty(ml * Lr, H, device=dev, dtype=torch.bfloat16)
            o.gemm(logits, st.model.head_weight(), dhr, False, True)              # d h = dLogits W_head
            o.gemm(logits, hr, st.model.head_grad(), True, True, accumulate=True, split_k=1)
            st.values_backward(hr, dv, dhr)
            dhf = torch.zeros(ml * cfg.seq_len, H, device=dev, dtype=torch.bfloat16)
            dhf.index_copy_(0, rows, dhr)
            dx = torch.empty_like(x_out)
            o.rmsnorm_bwd(dhf, x_out, st.model.f32["norm"], rstd, dx, None, st.model.g["norm"])
            return dx

        self._pass(st, seqs, True, loss_last)
        if self.tied and (st.first or st.last):
            dist.all_reduce(st.model.g["embed"], group=self.embed_group)
        st.step()
        torch.cuda.synchronize(dev)
        t_end = time.perf_counter()
        self.step_count += 1
        out = {"sync_s": t_sync - t0, "rollout_s": t_roll - t_sync, "score_s": t_score - t_roll,
               "train_s": t_end - t_score, "step_s": t_end - t0, "train_tokens": B * cfg.seq_len}
        # the last stage owns the losses and rewards: share them
        vec = torch.zeros(6, device=dev)
        if st.last:
            if self.tp > 1:
                dist.all_reduce(stats, group=self.tp_group)
            vec[:4] = stats
            vec[4] = seq_reward.mean()
            vec[5] = (old_lp - ref_lp).mean()
        dist.broadcast(vec, src=self.ranks[-1], group=self.group)
        v = vec.tolist()
        out.update({"pg_loss": v[0], "vf_loss": v[1], "clipfrac": v[2] / max(v[3], 1.0), "reward_mean": v[4],
                    "kl": v[5]})
        return out
