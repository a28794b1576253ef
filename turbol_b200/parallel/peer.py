"""Symmetric NVLink peer memory and the fused data-parallel optimizer step.

:class:`PeerBuffers` allocates one buffer per rank (``turbol_core.ops.PeerMemory``),
exchanges the CUDA IPC handles through the process group, and maps every
peer's buffer, so the kernels in ``csrc/kernels/comm.cu`` read and write peer
HBM directly over NVLink.

:class:`FusedDataParallelAdam` keeps a model's flat fp32 weights, flat fp32
gradient and bf16 weight copy inside that symmetric memory; one kernel per step
reduces the gradient across ranks, runs Adam on the shard each rank owns (the
Adam moments are allocated for that shard only: ZeRO-1) and
writes the updated weights (fp32 and bf16) into every rank.  It replaces
"NCCL all-reduce + local Adam" with a single launch that is replayable inside a
CUDA graph.  :class:`FusedGradSync` is the gradient-only variant (sum/mean
all-reduce of a flat buffer) with the trainer's ``grad_sync`` interface.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._native import ops as _ops


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


class PeerBuffers:
    def __init__(self, payload_bytes: int, group=None, device=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        dev = device if device is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", dev) if isinstance(dev, int) else torch.device(dev)
        self.mem = _ops().PeerMemory(int(payload_bytes), self.device.index)
        handles = [None] * self.world
        dist.all_gather_object(handles, self.mem.handle(), group=group)
        self.mem.open(handles, self.rank)
        dist.barrier(group=group)

    def tensor(self, offset: int, numel: int, dtype) -> torch.Tensor:
        return self.mem.tensor(offset, numel, dtype)

    def check(self):
        e = self.mem.error()
        if e:
            self.mem.clear_error()
            raise RuntimeError(f"peer-memory collective timed out waiting on a peer (site {e})")


# The replicated one-handshake step is offered for vectors up to this size
# (its moments are full-size on every rank).  It is opt-in: on two B200s,
# inside the PPO minibatch graph (144,448 parameters), it measured 25.7 µs per
# call against 20 µs for the ZeRO-1 kernel.
REPLICATED_MAX_NUMEL = 1 << 22


class FusedDataParallelAdam:
    """Owns flat (param fp32, grad fp32, bf16 shadow) tensors in peer memory.

    ``replicated=True`` (vectors up to REPLICATED_MAX_NUMEL): every rank pulls
    every peer's gradient and updates the whole vector itself, one handshake
    per call and no weights over NVLink (``allreduce_adam_rep``).  Default:
    ZeRO-1 (``allreduce_adam``: each rank updates its shard, the moments exist
    for that shard only, and the weights are all-gathered in the same kernel)."""

    capturable = True
    kernels_per_call = 1

    def __init__(self, numel: int, group=None, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                 replicated: bool = False):
        self.numel = int(numel)
        self.replicated = bool(replicated)
        if self.replicated and self.numel > REPLICATED_MAX_NUMEL:
            raise ValueError(f"replicated data-parallel Adam is for vectors up to {REPLICATED_MAX_NUMEL} parameters")
        n4 = _align(self.numel * 4)
        n2 = _align(self.numel * 2)
        self.off_param, self.off_grad, self.off_shadow = 0, n4, 2 * n4
        self.off_send = 2 * n4 + n2  # replicated: the gradient snapshot the peers read
        self.pb = PeerBuffers(2 * n4 + n2 + (n4 if self.replicated else 0), group)
        self.world = self.pb.world
        self.param = self.pb.tensor(self.off_param, self.numel, torch.float32)
        self.grad = self.pb.tensor(self.off_grad, self.numel, torch.float32)
        self.shadow = self.pb.tensor(self.off_shadow, self.numel, torch.bfloat16)
        dev = self.param.device
        if self.replicated:
            self.shard_lo, self.shard_hi = 0, self.numel
        else:
            # ZeRO-1: the Adam moments exist only for the slice this rank updates
            self.shard_lo, self.shard_hi = _ops().peer_owned_slice(self.numel, self.pb.rank, self.world)
        shard = max(1, self.shard_hi - self.shard_lo)
        self.m = torch.zeros(shard, device=dev)
        self.v = torch.zeros(shard, device=dev)
        self.step_t = torch.zeros(1, dtype=torch.int64, device=dev)
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.scale = 1.0 / self.world

    def broadcast_params(self, src: int = 0):
        """Makes every rank start from the weights of rank ``src`` of the group."""
        g = self.pb.group
        dist.broadcast(self.param, src=dist.get_global_rank(g, src) if g is not None else src, group=g)
        self.shadow.copy_(self.param)
        torch.cuda.synchronize()

    def step(self, grad_scale: float = None):
        gs = self.scale if grad_scale is None else grad_scale
        if self.replicated:
            self.pb.mem.allreduce_adam_rep(self.off_grad, self.off_send, self.off_param, self.off_shadow, self.numel,
                                           self.m, self.v, self.lr, self.betas[0], self.betas[1], self.eps, self.wd,
                                           gs, self.step_t)
        else:
            self.pb.mem.allreduce_adam(self.off_grad, self.off_param, self.off_shadow, self.numel, self.m, self.v,
                                       self.lr, self.betas[0], self.betas[1], self.eps, self.wd, gs, self.step_t)
        _ops().counter_add(self.step_t, 1)

    def state_dict(self):
        """This rank's optimizer state: the moments of elements [lo, hi) of the
        flat parameter vector (ZeRO-1: its shard; replicated: the whole vector;
        each data-parallel rank saves its own)."""
        return {"m": self.m, "v": self.v, "step": self.step_t.clone(), "shard": (self.shard_lo, self.shard_hi),
                "numel": self.numel, "world": self.world}

    def load_state_dict(self, sd):
        shard = tuple(sd.get("shard", (self.shard_lo, self.shard_hi)))
        if shard != (self.shard_lo, self.shard_hi) or sd["m"].numel() != self.m.numel():
            raise ValueError(f"optimizer shard {shard} does not match this rank's slice "
                             f"({self.shard_lo}, {self.shard_hi}); load the file saved by the same data-parallel rank")
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        self.step_t.copy_(sd["step"])

    def check(self):
        self.pb.check()


class FusedGradSync:
    """All-reduce (mean) of a flat fp32 gradient through peer memory.

    ``bind(flat_grad)`` is not needed: the trainer asks for the buffer with
    :meth:`allocate` so the gradient is produced in symmetric memory."""

    capturable = True
    kernels_per_call = 1

    def __init__(self, group=None, max_numel: int = 1 << 24):
        self.group = group
        self.world = dist.get_world_size(group)
        self.scale = 1.0 / self.world
        self.max_numel = max_numel
        self.pb = None
        self.buf = None

    def allocate(self, numel: int) -> torch.Tensor:
        self.pb = PeerBuffers(_align(numel * 4), self.group)
        self.buf = self.pb.tensor(0, numel, torch.float32)
        return self.buf

    def __call__(self, flat_grad: torch.Tensor) -> float:
        if self.buf is None or flat_grad.data_ptr() != self.buf.data_ptr():
            raise RuntimeError("FusedGradSync: the gradient must live in the buffer from allocate()")
        self.pb.mem.allreduce(0, 0, flat_grad.numel(), 1.0)
        return self.scale

    def check(self):
        if self.pb is not None:
            self.pb.check()
