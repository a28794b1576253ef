"""Worker for the tensor-parallel fused-kernel tests (launched by
test_tp_multigpu.py under torch.distributed.run, one process per GPU).
Checks all-gather->GEMM and GEMM->reduce-scatter against NCCL collectives +
fp32 matmuls, several calls in a row (both buffer halves, interleaved), then
times both against the unfused NCCL path.  Exits non-zero on a mismatch."""
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200._native import ops  # noqa: E402
from turbol_b200.parallel.tp import TensorParallelComm  # noqa: E402


def rnd(shape, seed, dev, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dev, torch.bfloat16)


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    o = ops()
    tp = TensorParallelComm(max_rows=8192, max_in=2048, max_out=2048)
    for it, (mloc, K, N, bmn) in enumerate([(256, 1536, 1024, False), (3072, 1536, 2048, False),
                                             (128, 512, 384, True), (256, 1536, 1024, False)]):
        M = mloc * world
        Wt = rnd((K, N) if bmn else (N, K), 1000 + 10 * it + rank, dev, 0.05)
        Wf = Wt.float() if bmn else Wt.float().t()
        for rep in range(3):  # new inputs every call: stale buffers would show
            # ---- all-gather -> GEMM
            shard = rnd((mloc, K), 100 * it + 10 * rep + rank, dev)
            full = [torch.empty_like(shard) for _ in range(world)]
            dist.all_gather(full, shard)
            ref = torch.cat(full).float() @ Wf
            y = tp.all_gather_gemm(shard, Wt, b_mn=bmn)
            torch.cuda.synchronize()
            err = (y.float() - ref).abs().max().item()
            assert err < 0.02 * ref.abs().max().item() + 1e-3, ("ag", it, rep, err)
            # ---- GEMM -> reduce-scatter (+ residual), interleaved with all-gathers
            A = rnd((M, K), 200 * it + 10 * rep + rank, dev)
            res = rnd((mloc, N), 300 * it + 10 * rep + rank, dev)
            tot = A.float() @ Wf
            dist.all_reduce(tot)
            exp = tot[rank * mloc:(rank + 1) * mloc] + res.float()
            out = tp.gemm_reduce_scatter(A, Wt, b_mn=bmn, residual=res)
            y2 = tp.all_gather_gemm(shard, Wt, b_mn=bmn)
            torch.cuda.synchronize()
            err = (out.float() - exp).abs().max().item()
            assert err < 0.02 * exp.abs().max().item() + 1e-2, ("rs", it, rep, err)
            assert torch.equal(y2, y), ("ag repeat", it, rep)
            tp.check()
        tp.check()
    # ---- timing at a training shape: fused vs NCCL + GEMM (max over ranks)
    mloc, K, N = 3072, 1536, 2048
    M = mloc * world
    shard = rnd((mloc, K), 7 + rank, dev)
    W1 = rnd((N // world, K), 8 + rank, dev, 0.05)   # column-parallel: N split across ranks
    A = rnd((M, K // world), 9 + rank, dev)
    W2 = rnd((N, K // world), 10 + rank, dev, 0.05)  # row-parallel: K split across ranks
    gbuf = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
    y = torch.empty(M, N // world, device=dev, dtype=torch.bfloat16)
    yp = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    rs_out = torch.empty(mloc, N, device=dev, dtype=torch.bfloat16)

    def t(fn, n=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b) / n], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item()

    ag_fused = t(lambda: tp.all_gather_gemm(shard, W1, out=y))
    ag_nccl = t(lambda: (dist.all_gather_into_tensor(gbuf, shard), o.gemm(gbuf, W1, y)))
    gemm_only_ag = t(lambda: o.gemm(gbuf, W1, y))
    rs_fused = t(lambda: tp.gemm_reduce_scatter(A, W2, out=rs_out))
    rs_nccl = t(lambda: (o.gemm(A, W2, yp), dist.reduce_scatter_tensor(rs_out, yp)))
    gemm_only_rs = t(lambda: o.gemm(A, W2, yp))
    tp.check()
    if rank == 0:
        # roofline: max(GEMM time at the measured peak, NVLink bytes at 770 GB/s per direction)
        peak = 1615.3e12
        ag_flops = 2.0 * M * (N // world) * K
        ag_bytes = (world - 1) * mloc * K * 2
        rs_flops = 2.0 * M * N * (K // world)
        rs_bytes = (world - 1) * mloc * N * 2
        ag_roof = max(ag_flops / peak, ag_bytes / 770e9) * 1e3
        rs_roof = max(rs_flops / peak, rs_bytes / 770e9) * 1e3
        print(json.dumps({"world": world, "shape": {"rows_per_rank": mloc, "K": K, "N": N},
                          "ag_gemm_ms": {"fused": ag_fused, "nccl_plus_gemm": ag_nccl, "gemm_only": gemm_only_ag,
                                         "roofline_ms": ag_roof, "frac_of_roofline": ag_roof / ag_fused},
                          "gemm_rs_ms": {"fused": rs_fused, "gemm_plus_nccl": rs_nccl, "gemm_only": gemm_only_rs,
                                         "roofline_ms": rs_roof, "frac_of_roofline": rs_roof / rs_fused}}))
        print("TP_WORKER_OK")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
