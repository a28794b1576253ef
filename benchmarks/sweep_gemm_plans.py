#!/usr/bin/env python
"""Tile-plan sweep of the tcgen05 GEMM on the shapes of a GRPO step (one GPU).

  python benchmarks/sweep_gemm_plans.py [--model qwen2-1.5b|llama3-8b] [--batch 512] [--tokens 6144]

For every shape it times the automatic plan and each (tile width BN, split-K)
pair the kernel accepts, as CUDA-graph replays cycling through per-layer weight
copies (so weights stream from HBM as in a real step), and prints the best
plan next to the automatic one and cuBLAS (torch.matmul, the library baseline,
forward shapes only).  Shapes:

* decode projections at M = batch rows (the rollout engine's step);
* training weight gradients dW[out, in] += dY^T X over `tokens` rows (both
  operands MN-major, fp32 accumulation), the GEMMs the hand-written backward
  issues once per layer and micro-batch.
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200._native import ops  # noqa: E402
from turbol_b200.models.llm import LMConfig  # noqa: E402


def graph_us(fn, reps=8):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / reps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2-1.5b", choices=["qwen2-1.5b", "llama3-8b"])
    ap.add_argument("--batch", type=int, default=512)
    ap.add_argument("--tokens", type=int, default=6144)
    ap.add_argument("--copies", type=int, default=4)
    a = ap.parse_args()
    cfg = LMConfig.qwen2_1p5b() if a.model == "qwen2-1.5b" else LMConfig.llama3_8b()
    o = ops()
    dev = torch.device("cuda", 0)
    H, F = cfg.hidden, cfg.ffn
    out = {"model": a.model, "decode": {}, "weight_grad": {}}
    # ---- decode projections: C[M, N] = X[M, K] . W[N, K]^T
    M = a.batch
    for name, N, K in (("qkv", cfg.qkv_dim, H), ("o", H, cfg.q_dim), ("gate_up", 2 * F, H), ("down", H, F),
                       ("lm_head", cfg.vocab, H)):
        Ws = [(torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16) for _ in range(a.copies)]
        X = torch.randn(M, K, device=dev).to(torch.bfloat16)
        C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        ws = torch.zeros(max(o.gemm_workspace_numel(M, N, K) * 4, 1 << 20), device=dev)
        row = {"auto": graph_us(lambda: [o.gemm(X, W, C) for W in Ws]) / a.copies,
               "cublas": graph_us(lambda: [torch.matmul(X, W.t(), out=C) for W in Ws]) / a.copies}
        for bn in (64, 128, 256):
            for sk in (1, 2, 3, 4, 6, 8):
                try:
                    kw = {"bn": bn, "split_k": sk}
                    if sk > 1:
                        kw["workspace"] = ws
                    row[f"bn{bn}_s{sk}"] = graph_us(lambda: [o.gemm(X, W, C, **kw) for W in Ws]) / a.copies
                except Exception as e:  # a plan the kernel rejects
                    row[f"bn{bn}_s{sk}"] = None
        best = min((v, k) for k, v in row.items() if v is not None and k != "cublas")
        print(f"decode {name:8s} M={M} N={N} K={K}: auto {row['auto']:7.1f} us  best {best[1]} {best[0]:7.1f} us  "
              f"cuBLAS {row['cublas']:7.1f} us", flush=True)
        out["decode"][name] = row
        del Ws
    # ---- weight gradients: dW[N_out, K_in] += dY[T, N_out]^T X[T, K_in]
    T = a.tokens
    for name, Nout, Kin in (("qkv", cfg.qkv_dim, H), ("o", H, cfg.q_dim), ("gate_up", 2 * F, H), ("down", H, F)):
        dY = torch.randn(T, Nout, device=dev).to(torch.bfloat16)
        Xs = [torch.randn(T, Kin, device=dev).to(torch.bfloat16) for _ in range(2)]
        Gs = [torch.zeros(Nout, Kin, device=dev) for _ in range(2)]
        row = {"auto": graph_us(lambda: [o.gemm(dY, X, G, True, True, accumulate=True) for X, G in zip(Xs, Gs)]) / 2}
        for bn in (128, 256):
            for sk in (1, 2, 3):
                try:
                    row[f"bn{bn}_s{sk}"] = graph_us(lambda: [o.gemm(dY, X, G, True, True, accumulate=True, bn=bn,
                                                                    split_k=sk) for X, G in zip(Xs, Gs)]) / 2
                except Exception:
                    row[f"bn{bn}_s{sk}"] = None
        best = min((v, k) for k, v in row.items() if v is not None)
        fl = 2 * T * Nout * Kin
        print(f"dW     {name:8s} [{Nout}x{Kin}] K={T}: auto {row['auto']:7.1f} us ({fl / row['auto'] / 1e6:6.1f} TF/s)"
              f"  best {best[1]} {best[0]:7.1f} us ({fl / best[0] / 1e6:6.1f} TF/s)", flush=True)
        out["weight_grad"][name] = row
        del dY, Xs, Gs
    print(json.dumps(out))


if __name__ == "__main__":
    main()
