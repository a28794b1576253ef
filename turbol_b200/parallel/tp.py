"""Tensor parallelism with the collectives fused into the tcgen05 GEMM.

:class:`TensorParallelComm` owns one symmetric NVLink buffer per rank (CUDA
IPC, mapped into every peer) and exposes the two Megatron-style primitives
with the communication inside the GEMM kernel:

* ``all_gather_gemm(shard, W)`` - column-parallel input with sequence-sharded
  activations: ``Y[M, N_local] = concat_ranks(shard) . W_local^T``.  While a
  rank computes the tiles of its own rows, one warp per CTA pushes its shard
  into every peer's staging area with peer stores (16-byte vectors over
  NVLink) and raises one release flag per 32-row sub-chunk; a CTA that reaches
  a remote row tile waits (bounded) for that tile's flags and TMA-loads it from
  local staging, so each remote row crosses NVLink once.
* ``gemm_reduce_scatter(A, W)`` - row-parallel output:
  ``out[M/W, N] = (sum_ranks A_r . W_r^T)[this rank's rows] (+ bias) (+ residual)``.
  Every output tile is stored (bf16) straight from the GEMM epilogue into the
  receive slot of the rank that owns its rows, tile by tile as the GEMM runs;
  a short finishing kernel on each rank sums its slots once every CTA of every
  rank has arrived.

Reuse of the staging and receive areas alternates between two halves by the
parity of a device-side epoch, with "consumed" flags guarding the half that
a peer may still be reading, so consecutive calls need no host
synchronization and the calls can be captured in CUDA graphs.  Every wait is
bounded (4 s) and reports through an error word (:meth:`check`).
No TMA multicast is used anywhere: remote data moves by plain peer stores.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._native import ops as _ops
from .peer import PeerBuffers


def _align(x: int, a: int = 4096) -> int:
    return (x + a - 1) // a * a


class TensorParallelComm:
    def __init__(self, max_rows: int, max_in: int, max_out: int, group=None, device=None):
        """max_rows: the largest full row count M (all ranks' rows together);
        max_in: the largest K of an all-gather GEMM input; max_out: the largest N
        of a reduce-scatter GEMM output."""
        o = _ops()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.hdr_bytes = int(o.tp_header_bytes())
        self.ag_half = _align(max_rows * max_in * 2)
        self.rs_half = _align(max_rows * max_out * 2)
        self.ag_off = self.hdr_bytes
        self.rs_off = self.hdr_bytes + 2 * self.ag_half
        self.pb = PeerBuffers(self.rs_off + 2 * self.rs_half, group, device)
        self.device = self.pb.device
        with torch.cuda.device(self.device):
            self.pb.tensor(0, self.hdr_bytes // 4, torch.int32).zero_()
            self.ctr = torch.zeros(8, dtype=torch.int32, device=self.device)
            torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        self.max_rows, self.max_in, self.max_out = max_rows, max_in, max_out

    # ------------------------------------------------------------------ ops
    def all_gather_gemm(self, shard: torch.Tensor, W: torch.Tensor, out: torch.Tensor = None, b_mn: bool = False,
                        bias=None, aux=None, epi: int = 0, bn: int = 0, gather_out: torch.Tensor = None,
                        c2: torch.Tensor = None) -> torch.Tensor:
        """gather_out (optional, bf16 [M, K]): also receives the gathered rows
        (what the weight gradient of this projection needs in training).
        c2 (optional, bf16 [M, N], with the SwiGLU epilogue): also receives the
        raw gate/up product, which the SwiGLU backward needs."""
        M = shard.shape[0] * self.world
        K = shard.shape[1]
        N = W.shape[1] if b_mn else W.shape[0]
        if M > self.max_rows or K > self.max_in:
            raise ValueError("all_gather_gemm: shape beyond the communicator's capacity")
        if out is None:
            ncols = N // 2 if epi == _ops().EPI_SWIGLU else N
            out = torch.empty(M, ncols, device=shard.device, dtype=torch.bfloat16)
        self.pb.mem.tp_ag_gemm(0, self.ag_off, self.ag_half, self.ctr, shard, W, out, b_mn, bias, aux, epi, bn,
                               gather_out, c2)
        return out

    def gemm_reduce_scatter(self, A: torch.Tensor, W: torch.Tensor, out: torch.Tensor = None, b_mn: bool = False,
                            bias=None, residual=None, bn: int = 0) -> torch.Tensor:
        M = A.shape[0]
        N = W.shape[1] if b_mn else W.shape[0]
        if M > self.max_rows or N > self.max_out:
            raise ValueError("gemm_reduce_scatter: shape beyond the communicator's capacity")
        if out is None:
            out = torch.empty(M // self.world, N, device=A.device, dtype=torch.bfloat16)
        self.pb.mem.tp_gemm_rs(0, self.rs_off, self.rs_half, self.ctr, A, W, out, b_mn, bias, residual, bn)
        return out

    def check(self):
        """Raises if a bounded wait of a fused kernel ran out (synchronizes)."""
        e = int(self.ctr[6].item())
        if e:
            self.ctr[6].zero_()
            raise RuntimeError(f"tensor-parallel kernel timed out waiting on a peer (site {e})")
