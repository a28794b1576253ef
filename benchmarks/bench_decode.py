#!/usr/bin/env python
"""Decode-step kernel microbenchmarks (one GPU), timed as CUDA-graph replays.

  python benchmarks/bench_decode.py [--model qwen2-1.5b|llama3-8b] [--batch B] [--ctx C] [--only gemm|attn]

GEMMs: the per-layer projections of one decode step at M = batch rows (QKV
with bias, output with residual, gate/up with SwiGLU, down with residual) and
the LM head, cycling through every layer's weights (so weights stream from
HBM as in a real step), for the automatic tile plan and with a split-K
workspace.  Attention: paged GQA decode attention over `ctx` cached tokens,
with the prompt's 256 tokens shared by groups of 8 sequences.
"""
import argparse
import json
import math
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200._native import ops  # noqa: E402
from turbol_b200.models.llm import LMConfig  # noqa: E402


def graph_time(fn, reps=10):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
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
    ap.add_argument("--ctx", type=int, default=290)
    ap.add_argument("--only", default="all", choices=["all", "gemm", "attn"])
    ap.add_argument("--layers", type=int, default=0, help="layers to cycle through (default: the model's)")
    a = ap.parse_args()
    o = ops()
    dev = "cuda:0"
    cfg = LMConfig.qwen2_1p5b() if a.model == "qwen2-1.5b" else LMConfig.llama3_8b()
    L = a.layers or cfg.n_layers
    res = {"model": a.model, "batch": a.batch}
    if a.only in ("all", "attn"):
        G, bs, D = 8, 16, cfg.head_dim
        B = a.batch
        P = max(1, B // G)
        Lp = min(256, a.ctx)
        nb = (a.ctx + bs - 1) // bs
        npb = Lp // bs
        nblocks = P * npb + B * (nb - npb) + 1
        kcs = [torch.randn(nblocks, cfg.n_kv_heads, bs, D, device=dev).to(torch.bfloat16) for _ in range(L)]
        vcs = [torch.randn(nblocks, cfg.n_kv_heads, bs, D, device=dev).to(torch.bfloat16) for _ in range(L)]
        table = torch.zeros(B, nb, dtype=torch.int32)
        nxt = P * npb
        for s in range(B):
            p = s // G
            table[s, :npb] = torch.arange(p * npb, (p + 1) * npb)
            for j in range(npb, nb):
                table[s, j] = nxt
                nxt += 1
        table = table.to(dev)
        ctx = torch.full((B,), a.ctx, device=dev, dtype=torch.int32)
        q = torch.randn(B, cfg.qkv_dim, device=dev).to(torch.bfloat16)
        out = torch.empty(B, cfg.q_dim, device=dev, dtype=torch.bfloat16)

        def run():
            for li in range(L):
                o.decode_attention(q, kcs[li], vcs[li], table, ctx, out, cfg.n_heads, cfg.n_kv_heads, D, bs,
                                   1 / math.sqrt(D))
        us = graph_time(run) / L
        uniq = (P * npb + B * (nb - npb)) * cfg.n_kv_heads * bs * D * 4
        res["decode_attention_us"] = us
        res["decode_attention_unique_kv_gbs"] = uniq / us / 1e3
        print(f"decode attention B={B} ctx={a.ctx}: {us:.1f} us/layer, unique KV {uniq / 1e6:.1f} MB "
              f"-> {uniq / us / 1e3:.0f} GB/s")
        del kcs, vcs
    if a.only in ("all", "gemm"):
        M = a.batch
        shapes = {"qkv": (cfg.qkv_dim, cfg.hidden, o.EPI_BIAS if cfg.qkv_bias else o.EPI_NONE),
                  "o": (cfg.hidden, cfg.q_dim, o.EPI_RESIDUAL), "gate_up": (2 * cfg.ffn, cfg.hidden, o.EPI_SWIGLU),
                  "down": (cfg.hidden, cfg.ffn, o.EPI_RESIDUAL), "lm_head": (cfg.vocab, cfg.hidden, o.EPI_NONE)}
        res["gemm_us"] = {}
        for name, (N, K, epi) in shapes.items():
            nl = L if name != "lm_head" else 2
            Ws = [(torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16) for _ in range(nl)]
            A = torch.randn(M, K, device=dev).to(torch.bfloat16)
            C = torch.empty(M, N // 2 if epi == o.EPI_SWIGLU else N, device=dev, dtype=torch.bfloat16)
            aux = torch.randn(M, N, device=dev).to(torch.bfloat16)
            bias = torch.randn(N, device=dev)
            ws = torch.zeros(max(o.gemm_workspace_numel(M, N, K), 1), device=dev)
            row = {}
            # auto / split-k: the general tcgen05 GEMM; decode: the weight-stationary
            # decode GEMM (cluster split-K), not used for the LM head
            variants = [("auto", {}), ("split-k", {"workspace": ws})]
            if name != "lm_head":
                variants.append(("decode", None))
            for label, kw in variants:
                if epi == o.EPI_SWIGLU and kw and "workspace" in kw:
                    continue

                def run():
                    for W in Ws:
                        ep = {"bias": bias} if epi == o.EPI_BIAS else ({"aux": aux} if epi == o.EPI_RESIDUAL else {})
                        if kw is None:
                            o.gemm_decode(A, W, C, epi=epi, **ep)
                        else:
                            o.gemm(A, W, C, epi=epi, **ep, **kw)
                us = graph_time(run) / nl
                row[label] = us
                print(f"gemm {name:8s} M={M:5d} N={N:6d} K={K:5d} {label:8s} {us:8.1f} us  "
                      f"{2 * M * N * K / us / 1e6:7.1f} TF/s  weights {N * K * 2 / us / 1e3:6.0f} GB/s")
            res["gemm_us"][name] = row
            del Ws
    print(json.dumps(res))


if __name__ == "__main__":
    main()
