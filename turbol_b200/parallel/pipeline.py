"""Pipeline parallelism: 1F1B over NCCL point-to-point.

A :class:`PipelineStage` holds a contiguous block of decoder layers (the
first stage also the embedding, the last also the final norm, the LM head
and an optional value head) as a :class:`DecoderLM` slice with its own flat
fp32 master weights, gradient and bf16 copy.  :func:`run_1f1b` runs one
training step over ``M`` micro-batches with the one-forward-one-backward
schedule of PipeDream-Flush (Narayanan et al., "Efficient Large-Scale Language
Model Training on GPU Clusters Using Megatron-LM", SC'21): each stage does
``num_stages - stage - 1`` warm-up forwards, then alternates one forward and
one backward, then drains the remaining backwards, so at most
``num_stages - stage`` micro-batches of activations are alive per stage.
Activations go forward and their gradients backward with
``torch.distributed`` NCCL send/recv (with tensor parallelism inside the
stages, every rank sends its rows to the same TP rank of the next stage); a send to the next stage and the receive
from it are posted as one batched operation so the two directions never wait
on each other, and NCCL runs them on its own stream, overlapped with the next
micro-batch's compute.

The reference's ``PipelineTrainer`` (turbol_vllm/src/distributed/pipeline_trainer.cpp:55-145)
describes a GPipe schedule and executes it serially on one device; its
micro-batch order for 1F1B is the one ``turbol_core.PipelineSchedule`` returns.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch
import torch.distributed as dist

from .._native import ops as _ops
from ..models.llm import DecoderLM, LMConfig
from ..ops.rl import FusedAdam


def stage_layers(n_layers: int, num_stages: int, stage: int) -> List[int]:
    per = n_layers // num_stages
    extra = n_layers % num_stages
    lo = stage * per + min(stage, extra)
    return list(range(lo, lo + per + (1 if stage < extra else 0)))


class PipelineStage:
    VH_ROWS = 8  # the value head is a [1, H] linear layer stored as 8 rows (tile-friendly); row 0 is used

    def __init__(self, cfg: LMConfig, stage: int, num_stages: int, device, seed: int = 0, value_head: bool = False,
                 lr: float = 1e-5, betas=(0.9, 0.95), tp_comm=None, recompute: bool = False):
        """tp_comm: a :class:`TensorParallelComm` over this stage's
        tensor-parallel group; the stage then holds this rank's shard of its
        layers (:class:`TPTrainLM`) and its micro-batch rows are split over the
        group (each rank exchanges its rows with the same TP rank of the
        neighbouring stages).  recompute: activation recomputation in
        :func:`run_1f1b` (keep stage inputs only, re-run the forward before
        each backward)."""
        self.cfg, self.stage, self.num_stages = cfg, stage, num_stages
        self.recompute = recompute
        self.first, self.last = stage == 0, stage == num_stages - 1
        self.device = torch.device(device)
        self.tp_comm = tp_comm
        self.tp = tp_comm.world if tp_comm is not None else 1
        base = DecoderLM(cfg, self.device, layers=stage_layers(cfg.n_layers, num_stages, stage),
                         embed=self.first, head=self.last, seed=seed + 1009 * stage, master=tp_comm is None)
        if tp_comm is not None:
            from ..models.tp_llm import TPTrainLM

            self.model = TPTrainLM(base, tp_comm)
            del base
        else:
            self.model = base
        self.opt = FusedAdam(self.model.flat, self.model.grad, lr=lr, betas=betas, shadow=self.model.shadow)
        self.value_head = value_head and self.last
        if self.value_head:
            H = cfg.hidden
            self.vh = torch.zeros(self.VH_ROWS * H + 8, device=self.device)  # fp32 master [8, H] + bias
            g = torch.Generator(device=self.device).manual_seed(seed + 77)
            self.vh[:H].copy_(torch.randn(H, device=self.device, generator=g) * (1.0 / H ** 0.5))
            self.vh_grad = torch.zeros_like(self.vh)
            self.vh_bf16 = torch.zeros(self.VH_ROWS, H, device=self.device, dtype=torch.bfloat16)
            self.vh_opt = FusedAdam(self.vh, self.vh_grad, lr=lr, betas=betas)
            self.sync_value_head()

    def sync_value_head(self):
        H = self.cfg.hidden
        self.vh_bf16.copy_(self.vh[: self.VH_ROWS * H].view(self.VH_ROWS, H))

    @torch.no_grad()
    def load_from_full(self, full: DecoderLM):
        """Copies this stage's tensors (by name) from a full model (fp32 when it has master weights)."""
        if self.tp > 1:
            self.model.load_from(full)
            return
        src = full.p if full.flat is not None else full.s
        for name in self.model.offsets:
            self.model.p[name].copy_(src[name])
        self.model.sync_shadow()

    def zero_grad(self):
        self.model.zero_grad()
        if self.value_head:
            self.vh_grad.zero_()

    def step(self, grad_scale: float = 1.0):
        if self.tp > 1:  # replicated parameters saw only this rank's rows
            self.model.reduce_replicated_grads()
            if self.value_head:
                dist.all_reduce(self.vh_grad, group=self.tp_comm.group)
        self.opt.step(grad_scale)
        if self.value_head:
            self.vh_opt.step(grad_scale)
            self.sync_value_head()

    def values(self, h: torch.Tensor) -> torch.Tensor:
        """Value head on final-norm hidden rows h [R, H] -> [R] fp32."""
        o = _ops()
        out = torch.empty(h.shape[0], self.VH_ROWS, device=self.device)
        o.gemm(h, self.vh_bf16, out)
        return out[:, 0] + self.vh[self.VH_ROWS * self.cfg.hidden]

    def values_backward(self, h: torch.Tensor, dv: torch.Tensor, dh: torch.Tensor):
        """dv [R] -> accumulates the value-head gradient and adds dv * w into dh [R, H] (bf16)."""
        H = self.cfg.hidden
        w = self.vh[:H]
        self.vh_grad[:H] += (dv[:, None] * h.float()).sum(0)
        self.vh_grad[self.VH_ROWS * H] += dv.sum()
        dh.copy_((dh.float() + dv[:, None] * w[None, :]).to(torch.bfloat16))


class _P2P:
    """Batched NCCL send/recv between neighbouring stages."""

    def __init__(self, ranks: Sequence[int], stage: int, group=None):
        self.prev = ranks[stage - 1] if stage > 0 else None
        self.next = ranks[stage + 1] if stage + 1 < len(ranks) else None
        self.group = group
        self.pending: List = []  # (work, tensor) of sends in flight

    def exchange(self, send_next=None, send_prev=None, recv_next=None, recv_prev=None):
        ops = []
        if send_next is not None:
            ops.append(dist.P2POp(dist.isend, send_next, self.next, self.group))
        if send_prev is not None:
            ops.append(dist.P2POp(dist.isend, send_prev, self.prev, self.group))
        if recv_prev is not None:
            ops.append(dist.P2POp(dist.irecv, recv_prev, self.prev, self.group))
        if recv_next is not None:
            ops.append(dist.P2POp(dist.irecv, recv_next, self.next, self.group))
        if not ops:
            return
        works = dist.batch_isend_irecv(ops)
        for w in works:
            w.wait()  # stream-ordered: later kernels on this stream see the received data

    def drain(self):
        self.pending.clear()


def run_1f1b(stage: PipelineStage, ranks: Sequence[int], num_micro: int, micro_rows: int,
             forward_first: Callable[[int], torch.Tensor], loss_last: Callable[[int, torch.Tensor], torch.Tensor],
             backward_first: Callable[[int, torch.Tensor], None], group=None, forward_only: bool = False,
             recompute: Optional[bool] = None):
    """One pipeline pass over ``num_micro`` micro-batches of ``micro_rows``
    hidden rows each.

    recompute (default ``stage.recompute``): activation recomputation.  The
    forward keeps only each micro-batch's stage input; its backward first
    re-runs the stage forward from that input to rebuild the saved
    activations, then runs the backward.  A stage then holds one [rows, H]
    input per micro-batch in flight instead of every layer's activations, for
    one extra forward per micro-batch (the reference's
    ``PipelineConfig::activation_checkpointing``,
    turbol_vllm/include/turbol/distributed/pipeline_trainer.hpp:47).

    forward_first(i) -> x: the first stage's input rows of micro-batch i
    (the embedding).  loss_last(i, x_out) -> dx_out: on the last stage,
    computes the loss terms of micro-batch i from the stage output and returns
    d loss / d x_out (or None when ``forward_only``).  backward_first(i, dx_in):
    on the first stage, consumes the gradient w.r.t. its input (the
    embedding backward).  The caller's ``stage.model.forward`` needs
    micro-batch shapes through closures; here only rows matter."""
    H = stage.cfg.hidden
    dev = stage.device
    S, s = stage.num_stages, stage.stage
    p2p = _P2P(ranks, s, group)
    saved = {}
    shape = (micro_rows, H)

    def new():
        return torch.empty(shape, device=dev, dtype=torch.bfloat16)

    if recompute is None:
        recompute = getattr(stage, "recompute", False)

    def fwd(i, x_in):
        # with recompute the forward still saves (the same code path as the
        # recomputation, so the output sent on equals the rebuilt one) and drops
        # the activations at once: one micro-batch's worth exists at a time
        x_out, sv = stage_forward(stage, i, x_in, save=not forward_only)
        if not forward_only:
            saved[i] = (x_in, None if recompute else sv)
        return x_out

    def bwd(i, dx_out):
        x_in, sv = saved.pop(i)
        if sv is None:  # recompute: rebuild this micro-batch's activations from its input
            _, sv = stage_forward(stage, i, x_in, save=True)
        return stage_backward(stage, i, dx_out, sv)

    if forward_only:
        for i in range(num_micro):
            x_in = forward_first(i) if stage.first else None
            if not stage.first:
                x_in = new()
                p2p.exchange(recv_prev=x_in)
            x_out = fwd(i, x_in)
            if stage.last:
                loss_last(i, x_out)
            else:
                p2p.exchange(send_next=x_out)
        return

    warm = min(S - s - 1, num_micro)
    remaining = num_micro - warm
    fi = bi = 0
    # ---- warm-up forwards
    for _ in range(warm):
        x_in = forward_first(fi) if stage.first else new()
        if not stage.first:
            p2p.exchange(recv_prev=x_in)
        x_out = fwd(fi, x_in)
        p2p.exchange(send_next=x_out)
        fi += 1
    # ---- steady state: one forward, one backward
    x_in = None
    if remaining > 0:
        x_in = forward_first(fi) if stage.first else new()
        if not stage.first:
            p2p.exchange(recv_prev=x_in)
    for k in range(remaining):
        x_out = fwd(fi, x_in)
        fi += 1
        if stage.last:
            dx_out = loss_last(fi - 1, x_out)
        else:
            dx_out = new()
            p2p.exchange(send_next=x_out, recv_next=dx_out)
        dx_in = bwd(bi, dx_out)
        bi += 1
        last_iter = k == remaining - 1
        if last_iter:
            if stage.first:
                backward_first(bi - 1, dx_in)
            else:
                p2p.exchange(send_prev=dx_in)
        else:
            if stage.first:
                backward_first(bi - 1, dx_in)
                x_in = forward_first(fi)
            else:
                x_in = new()
                p2p.exchange(send_prev=dx_in, recv_prev=x_in)
    # ---- cool-down backwards
    for _ in range(warm):
        dx_out = new()
        p2p.exchange(recv_next=dx_out)
        dx_in = bwd(bi, dx_out)
        if stage.first:
            backward_first(bi, dx_in)
        else:
            p2p.exchange(send_prev=dx_in)
        bi += 1


# The stage computation: forward of this stage's layers with saved
# activations, and the matching backward.  The micro-batch geometry (B, T and
# positions) is bound by the trainer before the pass.
_GEOM = {}


def set_micro_geometry(B: int, T: int, pos: torch.Tensor):
    _GEOM["B"], _GEOM["T"], _GEOM["pos"] = B, T, pos


def stage_forward(stage: PipelineStage, i: int, x_in: torch.Tensor, save: bool):
    B, T, pos = _GEOM["B"], _GEOM["T"], _GEOM["pos"]
    if getattr(stage, "tp", 1) > 1:
        return stage.model.forward_train(x_in, B, T, pos, save=save)
    return stage.model.forward(x_in, B, T, pos, save=save)


def stage_backward(stage: PipelineStage, i: int, dx_out: torch.Tensor, saved):
    B, T, pos = _GEOM["B"], _GEOM["T"], _GEOM["pos"]
    return stage.model.backward(dx_out, saved, B, T, pos)
