#!/usr/bin/env python
"""The PPO actor-critic MLP's forward and backward alone (one GPU): the
minibatch GEMMs of bench.py's headline workload (32,768 rows, hidden 256 per
head, block-diagonal actor | critic) without the rest of the PPO step.

  python benchmarks/bench_mlp_step.py [--rows 32768] [--reps 50]

Prints the CUDA-event time of one forward + backward (the upstream gradient
is a fixed random tensor), and its bytes/FLOPs; a small, self-contained
command for ncu captures of these kernels.
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200.models.fused_mlp import PAD, FusedActorCritic  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=32768)
    ap.add_argument("--hidden", type=int, default=256)
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--no-variants", action="store_true", help="time the MLP step only (short runs for ncu)")
    ap.add_argument("--fused-head", action="store_true",
                    help="the PPO training step's path: hidden layers, then the one-pass output layer + clipped "
                         "loss + output-layer backward (ppo_head.cu), then the hidden backward")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    net = FusedActorCritic(4, 2, (a.hidden, a.hidden), device=dev, seed=0)
    B = a.rows
    ws = net.workspace(B)
    x = torch.zeros(B, PAD, device=dev, dtype=torch.bfloat16)
    x[:, :4] = torch.randn(B, 4, device=dev).to(torch.bfloat16)
    dout = (torch.randn(B, 2 * PAD, device=dev) * 1e-3).to(torch.bfloat16)

    act = torch.randint(0, 2, (B,), device=dev, dtype=torch.int32)
    old = torch.full((B,), -0.69, device=dev)
    adv = torch.randn(B, device=dev)
    ret = torch.randn(B, device=dev)
    stats = torch.zeros(8, device=dev)

    def step():
        if a.fused_head:
            net.forward_hidden(x, ws)
            net.loss_backward(x, ws, act, old, adv, ret, stats, 0.2, 0.5, 0.0)
            return
        net.forward(x, ws)
        ws["dout"].copy_(dout)
        net.grad.zero_()
        net.backward(x, ws)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(a.reps):
        step()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / a.reps
    H2 = 2 * a.hidden
    flops = 2 * B * (PAD * H2 + H2 * H2 + H2 * 2 * PAD) * 3
    res = {"benchmark": "ppo_mlp_fwd_bwd", "rows": B, "fused_head": a.fused_head, "us": us,
           "tflops": flops / us / 1e6, "activation_bytes_per_layer": B * H2 * 2}
    if a.no_variants:
        print(json.dumps(res))
        return
    # the three 8-wide pieces of the backward: tensor-core GEMM (+ split-K reduce)
    # against the CUDA-core two-pass kernels
    from turbol_b200._native import ops

    o = ops()
    S, G, H = net.s, net.g, a.hidden
    h2, h1, dz2, dz1, wsk = ws["h2"], ws["h1"], ws["dz2"], ws["dz1"], ws["splitk"]
    sc = torch.empty(o.skinny8_scratch_numel(H2), device=dev)

    def t(fn, reps=50):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    def dw3_gemm():
        for head, rows, cols in (("a", slice(0, PAD), slice(0, H)), ("c", slice(PAD, 2 * PAD), slice(H, 2 * H))):
            o.gemm(dout[:, rows], h2[:, cols], G["w3" + head], True, True, workspace=wsk)

    res["dW3_us"] = {"gemm": t(dw3_gemm), "cuda_core": t(lambda: o.skinny8_wgrad(h2, dout, G["w3"], H, 1, H2,
                                                                                 PAD * H2, False, sc))}
    res["dZ2_us"] = {"gemm": t(lambda: o.gemm(dout, S["w3"], dz2, False, True, aux=h2, epi=o.EPI_TANH_BWD,
                                              colsum=G["b2"])),
                     "cuda_core": t(lambda: o.mlp_head_dz(dout, h2, S["w3"], H, dz2, G["b2"], False, sc))}
    P = net.p
    res["out_fwd_us"] = {"gemm": t(lambda: o.gemm(h2, S["w3"], ws["out"], bias=P["b3"], epi=o.EPI_BIAS)),
                         "cuda_core": t(lambda: o.mlp_head_fwd(h2, S["w3"], P["b3"], H, ws["out"]))}
    # tile widths of the two K = 512 GEMMs (kg0: the whole K over a dense
    # block-diagonal W2; kgroup: each tile only its head's K range, reading the
    # packed diagonal blocks) and of the hidden-layer weight gradient
    w2_dense = torch.block_diag(S["w2a"], S["w2c"]).contiguous()
    for kg in (0, H):
        w2 = S["w2"] if kg else w2_dense
        for bn in (64, 128, 256):
            res[f"h2_fwd_kg{kg}_bn{bn}_us"] = t(lambda: o.gemm(h1, w2, h2, bias=P["b2"], epi=o.EPI_BIAS_TANH,
                                                               bn=bn, kgroup=kg))
            res[f"dZ1_kg{kg}_bn{bn}_us"] = t(lambda: o.gemm(dz2, w2, dz1, False, True, aux=h1,
                                                            epi=o.EPI_TANH_BWD, colsum=G["b1"], bn=bn, kgroup=kg))
    for bn in (128, 256):
        for sk in (0, 8, 16, 32):
            def dw2():
                for cols in (slice(0, H), slice(H, 2 * H)):
                    o.gemm(dz2[:, cols], h1[:, cols], G["w2a"], True, True, workspace=wsk, bn=bn, split_k=sk)
            try:
                res[f"dW2_bn{bn}_s{sk}_us"] = t(dw2)
            except Exception:
                res[f"dW2_bn{bn}_s{sk}_us"] = None
    for rows in (0, 64, 128, 256, 512):  # first layer: rows per CTA (0 = automatic)
        res[f"first_layer_rows{rows}_us"] = t(lambda: o.dense_k8_fwd(x, S["w1"], P["b1"], h1, True, rows))
    res["dW1_us"] = {"gemm": t(lambda: o.gemm(dz1, x, G["w1"], True, True, workspace=wsk)),
                     "cuda_core": t(lambda: o.skinny8_wgrad(dz1, x, G["w1"], H2, PAD, 1, 0, False, sc))}
    print(json.dumps(res))


if __name__ == "__main__":
    main()
