#!/usr/bin/env python
"""tcgen05 GEMM throughput against cuBLAS (torch.matmul, the library baseline).

  python benchmarks/bench_gemm.py [--shapes 8192x8192x8192,...] [--reps 20]

Every shape is C[M, N] = A[M, K] . B[N, K]^T in bf16 with fp32 accumulation
and bf16 output.  Inputs are rotated over enough copies to exceed the 126 MB
L2 between timed calls; CUDA events around `reps` calls after warm-up.
Prints one line per shape and a JSON summary.
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200._native import ops  # noqa: E402


def timed(fn, reps):
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    for i in range(reps):
        fn(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="8192x8192x8192,16384x17920x1536,6144x1536x8960,512x1536x1536")
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args()
    o = ops()
    res = []
    for sh in a.shapes.split(","):
        M, N, K = (int(x) for x in sh.split("x"))
        bytes_in = (M * K + N * K) * 2
        copies = max(1, min(8, (256 << 20) // max(bytes_in, 1) + 1))
        As = [torch.randn(M, K, device="cuda").to(torch.bfloat16) for _ in range(copies)]
        Bs = [torch.randn(N, K, device="cuda").to(torch.bfloat16) for _ in range(copies)]
        C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms = timed(lambda i: o.gemm(As[i % copies], Bs[i % copies], C), a.reps)
        ms_cublas = timed(lambda i: torch.matmul(As[i % copies], Bs[i % copies].t(), out=C), a.reps)
        tf, tfc = 2 * M * N * K / ms / 1e9, 2 * M * N * K / ms_cublas / 1e9
        print(f"{M}x{N}x{K}: tcgen05 {ms * 1e3:9.1f} us {tf:7.1f} TF/s | cuBLAS {ms_cublas * 1e3:9.1f} us {tfc:7.1f} TF/s")
        res.append({"M": M, "N": N, "K": K, "ms": ms, "tflops": tf, "cublas_ms": ms_cublas, "cublas_tflops": tfc})
        del As, Bs, C
    print(json.dumps({"benchmark": "gemm_bf16", "results": res}))


if __name__ == "__main__":
    main()
