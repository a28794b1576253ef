#!/usr/bin/env python
"""Tensor benchmark: the reference's benchmark_tensor
(turbol_vllm/benchmarks/benchmark_tensor.cpp:7-77) — 1000 creations and 1000
copies of a 1024×1024 fp32 tensor and one 100 MB copy — through this
framework's ``turbol_b200.Tensor`` on the host, plus the same copy on the
device (CUDA events) when a GPU is present.

    python benchmarks/benchmark_tensor.py
"""
from __future__ import annotations

import json
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import turbol_b200 as turbol  # noqa: E402


def host_ms(fn, iters):
    t0 = time.perf_counter()
    for _ in range(iters):
        fn()
    return (time.perf_counter() - t0) * 1e3


def main():
    res = {}
    it = 1000
    t = host_ms(lambda: turbol.Tensor([1024, 1024], "float32", "cpu"), it)
    res["creation_ms_per_iter"] = t / it
    src = turbol.Tensor([1024, 1024], "float32", "cpu")
    t = host_ms(lambda: src.clone(), it)
    res["copy_ms_per_iter"] = t / it
    n = 100 * 1024 * 1024 // 4
    big = turbol.from_torch(torch.ones(n))
    t = host_ms(lambda: big.clone(), 1)
    res["host_copy_100MB_GBps"] = 2 * n * 4 / (t / 1e3) / 1e9
    if torch.cuda.is_available():
        a = torch.ones(n, device="cuda")
        b = torch.empty_like(a)
        for _ in range(3):
            b.copy_(a)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(20):
            b.copy_(a)
        e1.record()
        torch.cuda.synchronize()
        res["device_copy_100MB_GBps"] = 2 * n * 4 / (e0.elapsed_time(e1) / 20 / 1e3) / 1e9
    for k, v in res.items():
        print(f"  {k:28s} {v:12.4f}")
    print(json.dumps({"benchmark": "tensor", "results": res}))


if __name__ == "__main__":
    main()
