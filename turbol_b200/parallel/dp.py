"""Data-parallel gradient reduction for flat gradient buffers.

Two implementations behind one callable interface
(``sync(flat_grad) -> scale`` plus ``scale``, ``capturable`` and
``kernels_per_call`` attributes, as the trainers expect):

* :class:`NcclGradSync` — ``torch.distributed.all_reduce`` (sum) on NCCL; the
  baseline path.  Not captured in CUDA graphs.
* :class:`FusedGradSync` — the product path: one kernel per call that reduces
  the flat gradient across ranks by reading every peer's buffer directly over
  NVLink (peer pointers from CUDA IPC), with bounded flag waits; capturable in
  CUDA graphs.  See :mod:`turbol_b200.parallel.peer`.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class NcclGradSync:
    capturable = False
    kernels_per_call = 0

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.scale = 1.0 / self.world

    def __call__(self, flat_grad: torch.Tensor) -> float:
        dist.all_reduce(flat_grad, op=dist.ReduceOp.SUM, group=self.group)
        return self.scale


def make_grad_sync(kind: str = "fused", group=None):
    if kind == "nccl":
        return NcclGradSync(group)
    if kind == "fused":
        from .peer import FusedGradSync

        return FusedGradSync(group)
    raise ValueError(f"unknown gradient sync {kind!r}")
