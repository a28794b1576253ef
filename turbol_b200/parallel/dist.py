"""Distributed runtime facade: the reference's ``DistributedConfig`` /
``DistributedTrainer`` API on ``torch.distributed`` (NCCL on GPUs, gloo on
CPU), plus the collectives and process-group mesh the trainers use.

Reference surface (turbol_vllm/include/turbol/distributed/distributed_trainer.hpp:7-34,
turbol_vllm/src/distributed/distributed_trainer.cpp:7-69, bound at
turbol_vllm/python/turbol/pybind11_bindings.cpp:358-374):

* ``DistributedConfig``: ``strategy, world_size, rank, master_addr,
  master_port, use_nccl``;
* ``DistributedTrainer(config)``: ``initialize, shutdown, all_reduce(tensor,
  op="sum"|"mean"), broadcast(tensor, root_rank=0), get_rank,
  get_world_size``; a no-op when ``world_size == 1``; every call returns a
  ``Status``.

Differences by design: each rank binds its own GPU (``LOCAL_RANK``, not
device 0 for every rank), ``mean`` divides on the device (no host round
trip), every tensor dtype is accepted (not only fp32), rendezvous and
collectives run under a timeout and report ``kTimeout`` instead of hanging,
and ``all_gather``, ``reduce_scatter``, ``send``, ``recv``, ``barrier`` and a
DP x TP x PP group mesh are added.  Tensors may be ``torch.Tensor`` or the
core ``Tensor`` (viewed zero-copy).
"""
from __future__ import annotations

import datetime
import enum
import os
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from .._native import core as _core


class ParallelStrategy(enum.IntEnum):
    kDataParallel = 0
    kModelParallel = 1
    kPipelineParallel = 2


@dataclass
class DistributedConfig:
    strategy: ParallelStrategy = ParallelStrategy.kDataParallel
    world_size: int = 1
    rank: int = 0
    master_addr: str = "127.0.0.1"
    master_port: int = 29500
    use_nccl: bool = False
    # additions
    local_rank: Optional[int] = None  # GPU index on this node (default: LOCAL_RANK or rank)
    timeout_s: float = 120.0          # rendezvous and collective timeout
    tp_size: int = 1                  # mesh: tensor-parallel group size (innermost)
    pp_size: int = 1                  # mesh: pipeline stages (outermost)

    @classmethod
    def from_env(cls, **overrides) -> "DistributedConfig":
        """Reads the torchrun variables RANK, WORLD_SIZE, LOCAL_RANK, MASTER_ADDR, MASTER_PORT."""
        env = os.environ
        cfg = cls(world_size=int(env.get("WORLD_SIZE", 1)), rank=int(env.get("RANK", 0)),
                  master_addr=env.get("MASTER_ADDR", "127.0.0.1"), master_port=int(env.get("MASTER_PORT", 29500)),
                  local_rank=int(env["LOCAL_RANK"]) if "LOCAL_RANK" in env else None,
                  use_nccl=torch.cuda.is_available())
        for k, v in overrides.items():
            setattr(cfg, k, v)
        return cfg


def _status(code: Optional[str] = None, msg: str = ""):
    c = _core()
    if code is None:
        return c.Status()
    return c.Status(getattr(c.StatusCode, code), msg)


def _as_torch(t) -> torch.Tensor:
    if isinstance(t, torch.Tensor):
        return t
    if hasattr(t, "torch"):
        return t.torch()  # core Tensor -> zero-copy view
    raise TypeError(f"expected a torch.Tensor or turbol Tensor, got {type(t).__name__}")


_OPS = {"sum": dist.ReduceOp.SUM, "mean": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN,
        "prod": dist.ReduceOp.PRODUCT}


@dataclass
class Mesh:
    """Process groups for a DP x TP x PP layout.  Rank r has tp = r % T,
    dp = (r // T) % D, pp = r // (T * D): tensor parallelism innermost (its
    collectives are the most frequent; on NVSwitch every pair of GPUs is
    equally connected, so placement only decides group sizes)."""
    tp: int
    dp: int
    pp: int
    tp_rank: int
    dp_rank: int
    pp_rank: int
    tp_group: object = None
    dp_group: object = None
    pp_group: object = None
    pp_ranks: List[int] = field(default_factory=list)  # global ranks of this rank's pipeline, by stage


def build_mesh(world: int, rank: int, tp: int = 1, pp: int = 1) -> Mesh:
    if world % (tp * pp):
        raise ValueError(f"world size {world} is not divisible by tp*pp = {tp * pp}")
    dp = world // (tp * pp)
    m = Mesh(tp=tp, dp=dp, pp=pp, tp_rank=rank % tp, dp_rank=(rank // tp) % dp, pp_rank=rank // (tp * dp))
    if not dist.is_initialized():
        return m
    # every rank must create every group, in the same order
    for p in range(pp):
        for d in range(dp):
            ranks = [p * tp * dp + d * tp + t for t in range(tp)]
            g = dist.new_group(ranks)
            if rank in ranks:
                m.tp_group = g
    for p in range(pp):
        for t in range(tp):
            ranks = [p * tp * dp + d * tp + t for d in range(dp)]
            g = dist.new_group(ranks)
            if rank in ranks:
                m.dp_group = g
    for d in range(dp):
        for t in range(tp):
            ranks = [p * tp * dp + d * tp + t for p in range(pp)]
            g = dist.new_group(ranks)
            if rank in ranks:
                m.pp_group = g
                m.pp_ranks = ranks
    return m


class DistributedTrainer:
    def __init__(self, config: Optional[DistributedConfig] = None):
        self.config = config or DistributedConfig()
        self.initialized = False
        self._owns_group = False
        self.mesh: Optional[Mesh] = None

    # ------------------------------------------------------------ lifecycle
    @property
    def device(self) -> torch.device:
        c = self.config
        if c.use_nccl and torch.cuda.is_available():
            lr = c.local_rank if c.local_rank is not None else c.rank % max(torch.cuda.device_count(), 1)
            return torch.device("cuda", lr)
        return torch.device("cpu")

    def initialize(self):
        c = self.config
        if self.initialized:
            return _status()
        if c.world_size < 1 or not (0 <= c.rank < c.world_size):
            return _status("kInvalidArgument", f"rank {c.rank} / world_size {c.world_size}")
        if c.world_size == 1:
            self.initialized = True
            self.mesh = build_mesh(1, 0, 1, 1)
            return _status()
        try:
            if not dist.is_initialized():
                backend = "nccl" if (c.use_nccl and torch.cuda.is_available()) else "gloo"
                if backend == "nccl":
                    torch.cuda.set_device(self.device)
                dist.init_process_group(backend, init_method=f"tcp://{c.master_addr}:{c.master_port}",
                                        rank=c.rank, world_size=c.world_size,
                                        timeout=datetime.timedelta(seconds=c.timeout_s))
                self._owns_group = True
            elif dist.get_world_size() != c.world_size or dist.get_rank() != c.rank:
                return _status("kInvalidArgument", "an existing process group has a different rank / world size")
            self.mesh = build_mesh(c.world_size, c.rank, c.tp_size, c.pp_size)
        except (RuntimeError, ValueError) as e:
            code = "kTimeout" if "timed out" in str(e).lower() or "timeout" in str(e).lower() else "kUnavailable"
            return _status(code, str(e))
        self.initialized = True
        return _status()

    def shutdown(self):
        if self._owns_group and dist.is_initialized():
            dist.destroy_process_group()
        self._owns_group = False
        self.initialized = False
        return _status()

    def get_rank(self) -> int:
        return self.config.rank

    def get_world_size(self) -> int:
        return self.config.world_size

    # ------------------------------------------------------------ collectives
    def _run(self, fn):
        if not self.initialized:
            return _status("kUnavailable", "DistributedTrainer is not initialized")
        if self.config.world_size == 1:
            return _status()
        try:
            fn()
        except RuntimeError as e:
            code = "kTimeout" if "timeout" in str(e).lower() or "timed out" in str(e).lower() else "kInternalError"
            return _status(code, str(e))
        return _status()

    def all_reduce(self, tensor, op: str = "sum", group=None):
        if op not in _OPS:
            return _status("kInvalidArgument", f"unknown reduce op {op!r}")
        t = _as_torch(tensor)

        def go():
            dist.all_reduce(t, op=_OPS[op], group=group)
            if op == "mean":
                t.div_(dist.get_world_size(group))
        return self._run(go)

    def broadcast(self, tensor, root_rank: int = 0, group=None):
        t = _as_torch(tensor)
        return self._run(lambda: dist.broadcast(t, src=root_rank, group=group))

    def all_gather(self, output, tensor, group=None):
        """output: a tensor of world x tensor's size (concatenated along dim 0) or a list of tensors."""
        t = _as_torch(tensor)
        if isinstance(output, (list, tuple)):
            outs = [_as_torch(o) for o in output]
            return self._run(lambda: dist.all_gather(outs, t, group=group))
        o = _as_torch(output)
        return self._run(lambda: dist.all_gather_into_tensor(o, t, group=group))

    def reduce_scatter(self, output, tensor, op: str = "sum", group=None):
        """tensor: world x output's size along dim 0; rank r receives chunk r reduced."""
        if op not in ("sum", "mean", "max", "min"):
            return _status("kInvalidArgument", f"unknown reduce op {op!r}")
        o, t = _as_torch(output), _as_torch(tensor)

        def go():
            dist.reduce_scatter_tensor(o, t, op=_OPS[op], group=group)
            if op == "mean":
                o.div_(dist.get_world_size(group))
        return self._run(go)

    def send(self, tensor, dst: int, group=None):
        t = _as_torch(tensor)
        return self._run(lambda: dist.send(t, dst, group=group))

    def recv(self, tensor, src: int, group=None):
        t = _as_torch(tensor)
        return self._run(lambda: dist.recv(t, src, group=group))

    def barrier(self, group=None):
        def go():
            if self.device.type == "cuda":
                dist.barrier(group=group, device_ids=[self.device.index])
            else:
                dist.barrier(group=group)
        return self._run(go)


def initialize_from_env(**overrides) -> DistributedTrainer:
    """Convenience: a DistributedTrainer for a torchrun-launched process, initialized."""
    tr = DistributedTrainer(DistributedConfig.from_env(**overrides))
    st = tr.initialize()
    if not st.ok():
        raise RuntimeError(f"distributed initialization failed: {st}")
    return tr


__all__: Sequence[str] = ("ParallelStrategy", "DistributedConfig", "DistributedTrainer", "Mesh", "build_mesh",
                          "initialize_from_env")
