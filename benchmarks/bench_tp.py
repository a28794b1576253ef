#!/usr/bin/env python
"""Fused tensor-parallel GEMM collectives vs NCCL + GEMM, with roofline.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 benchmarks/bench_tp.py [--model llama3-8b|qwen2-1.5b|all]

Times, per projection of one decoder layer at the training micro-batch
(rows = sequences x tokens), the two fused kernels of ``TensorParallelComm``:

* all-gather -> GEMM (column parallel: QKV and gate/up; the sequence-sharded
  activation is gathered inside the GEMM kernel);
* GEMM -> reduce-scatter (row parallel: O and down projections, with the
  residual added in the finishing pass);

against the unfused path (NCCL all_gather_into_tensor / reduce_scatter_tensor
+ the same tcgen05 GEMM) and the GEMM alone.  Roofline per call = max(GEMM
FLOPs / measured bf16 peak, bytes that cross NVLink / 770 GB/s per direction);
the JSON line reports achieved / roofline.  CUDA-event times, mean of
``--iters`` back-to-back calls after 3 warm-ups, max over ranks.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200._native import ops  # noqa: E402
from turbol_b200.parallel.tp import TensorParallelComm  # noqa: E402

# (rows of the micro-batch, hidden, q+2kv projection width, ffn)
MODELS = {
    "llama3-8b": dict(rows=4 * 1536, hidden=4096, qkv=4096 + 2 * 1024, ffn=14336),
    "qwen2-1.5b": dict(rows=8 * 768, hidden=1536, qkv=1536 + 2 * 256, ffn=8960),
}
LINK_GBS = 770e9


def peak_flops():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]) * 1e12, "measured"
    except (OSError, KeyError, ValueError):
        return 1.59e15, "fallback"


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model", default="all", choices=["all"] + list(MODELS))
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", local)
    o = ops()
    peak, peak_src = peak_flops()
    models = list(MODELS) if a.model == "all" else [a.model]
    max_rows = max(MODELS[m]["rows"] for m in models)
    max_in = max(MODELS[m]["hidden"] for m in models)
    max_out = max_in
    tp = TensorParallelComm(max_rows, max_in, max_out, device=dev)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)

    def rnd(*shape, s=0.5):
        return (torch.randn(*shape, device=dev, generator=g) * s).to(torch.bfloat16)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / a.iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    results = []
    for name in models:
        m = MODELS[name]
        M, H = m["rows"], m["hidden"]
        mloc = M // world
        # column parallel: N split over ranks; row parallel: K split over ranks
        cases = [("qkv", "ag", H, m["qkv"]), ("gate_up", "ag", H, 2 * m["ffn"]),
                 ("o", "rs", H, H), ("down", "rs", m["ffn"], H)]
        for proj, kind, K, N in cases:
            if kind == "ag":
                Nl = N // world
                shard, W = rnd(mloc, K), rnd(Nl, K, s=0.02)
                y = torch.empty(M, Nl, device=dev, dtype=torch.bfloat16)
                gbuf = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
                fused = timed(lambda: tp.all_gather_gemm(shard, W, out=y))
                yf = y.clone()
                unfused = timed(lambda: (dist.all_gather_into_tensor(gbuf, shard), o.gemm(gbuf, W, y)))
                gemm = timed(lambda: o.gemm(gbuf, W, y))
                diff = (yf.float() - y.float()).abs().max().item() / (y.float().abs().max().item() + 1e-6)
                flops = 2.0 * M * Nl * K
                link = (world - 1) * mloc * K * 2
            else:
                Kl = K // world
                A, W = rnd(M, Kl), rnd(N, Kl, s=0.02)
                res = rnd(mloc, N)
                out = torch.empty(mloc, N, device=dev, dtype=torch.bfloat16)
                yp = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                fused = timed(lambda: tp.gemm_reduce_scatter(A, W, out=out, residual=res))
                of = out.float() - res.float()
                unfused = timed(lambda: (o.gemm(A, W, yp), dist.reduce_scatter_tensor(out, yp)))
                gemm = timed(lambda: o.gemm(A, W, yp))
                diff = (of - out.float()).abs().max().item() / (out.float().abs().max().item() + 1e-6)
                flops = 2.0 * M * N * Kl
                link = (world - 1) * mloc * N * 2
            roof = max(flops / peak, link / LINK_GBS) * 1e3
            results.append({"model": name, "proj": proj, "op": "all_gather_gemm" if kind == "ag" else
                            "gemm_reduce_scatter", "M": M, "K": K, "N": N, "fused_ms": fused,
                            "nccl_plus_gemm_ms": unfused, "gemm_only_ms": gemm, "roofline_ms": roof,
                            "frac_of_roofline": roof / fused, "speedup_vs_nccl": unfused / fused,
                            "max_rel_diff_vs_nccl": diff})
            if rank == 0:
                r = results[-1]
                print(f"{name:11s} {proj:8s} {r['op']:20s} M={M:6d} K={K:6d} N={N:6d}  fused {fused * 1e3:8.1f} us  "
                      f"nccl+gemm {unfused * 1e3:8.1f} us  gemm {gemm * 1e3:8.1f} us  roofline {roof * 1e3:8.1f} us  "
                      f"-> {roof / fused:.2f} of roofline  (max rel diff vs NCCL {diff:.1e})", flush=True)
    tp.check()
    if rank == 0:
        print(json.dumps({"benchmark": "tp_fused_collectives", "world": world, "peak_tflops": peak / 1e12,
                          "peak_source": peak_src, "link_gbs": LINK_GBS / 1e9,
                          "timing": "CUDA events, mean of back-to-back calls, max over ranks", "results": results}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
