#!/usr/bin/env python
"""Attention benchmark.

The reference's benchmark_attention (turbol_vllm/benchmarks/benchmark_attention.cpp:45-87)
prints the sizes of a (4, 8, 512, 64) problem and never launches a kernel.
This one times the framework's causal GQA flash attention (forward on
tcgen05 and on mma.sync, backward likewise; bf16, head_dim 128) at the
model shapes it serves, against
PyTorch's scaled_dot_product_attention on the same tensors (a library
kernel, for comparison only), and against the reference's own attention kernel
(turbol_vllm/src/cuda/attention.cu:16-97: fp32, one thread per query row,
non-causal, one K/V head per query head) when baseline/build_reference.sh has
compiled it into baseline/_ref/lib/libref_attention.so:

    python benchmarks/benchmark_attention.py [--steps 20] [--ref-steps 3]

The reference kernel runs on fp32 [B, H, T, D] copies of the same Q/K/V (K/V
heads repeated for GQA, every sequence at full length) and does the full
T x T product, twice the causal work; its time is reported as measured and
as a rate of that full work.

Shapes: the 1.5B GRPO training micro-batch (8 × 768 tokens, 12 query / 2 KV
heads) and the 8B PPO-RLHF micro-batch (4 × 1536 tokens, 32 / 8 heads).
Causal FLOPs: forward 2·B·Hq·T²·D (half of the dense 4·B·Hq·T²·D), backward
2.5× forward.  CUDA-event time, mean over --steps calls after 3 warm-ups.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import sys

import torch
import torch.nn.functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200._native import ops  # noqa: E402

REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref", "lib",
                       "libref_attention.so")
SHAPES = {"qwen2-1.5b train mb": (8, 768, 12, 2), "llama3-8b train mb": (4, 1536, 32, 8)}
D = 128


def timed(fn, steps):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def _ref_lib():
    if not os.path.exists(REF_LIB):
        return None
    lib = ctypes.CDLL(REF_LIB)
    f = lib.flash_attention_forward
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    return f


def bench_reference(qt, kt, vt, steps):
    """The reference kernel on fp32 [B, H, T, D] copies; returns (ms, max|diff| vs fp32 SDPA) or None."""
    f = _ref_lib()
    if f is None:
        return None
    B, H, T, Dh = qt.shape
    q, k, v = (t.float().contiguous() for t in (qt, kt, vt))
    out = torch.empty_like(q)
    lens = torch.full((B,), T, dtype=torch.int32, device=q.device)
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        rc = f(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lens.data_ptr(), B, H, T, Dh, stream)
        if rc != 0:
            raise RuntimeError(f"reference flash_attention_forward returned CUDA error {rc}")

    t = timed(call, steps)
    err = (out - F.scaled_dot_product_attention(q, k, v)).abs().max().item()
    return t, err


def bench_shape(name, B, T, Hq, Hk, steps, ref_steps=3):
    o = ops()
    dev = "cuda:0"
    ld = (Hq + 2 * Hk) * D
    qkv = (torch.randn(B * T, ld, device=dev) * 0.5).to(torch.bfloat16)
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D:(Hq + Hk) * D], qkv[:, (Hq + Hk) * D:]
    out = torch.empty(B * T, Hq * D, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(B * Hq * T, device=dev)
    delta = torch.empty_like(lse)
    dout = torch.randn_like(out)
    dqkv = torch.empty_like(qkv)
    scale = 1 / math.sqrt(D)
    fwd = lambda: o.flash_attn_fwd(q, k, v, out, lse, B, T, Hq, Hk, scale, impl="tc")  # noqa: E731
    fwd_mma = lambda: o.flash_attn_fwd(q, k, v, out, lse, B, T, Hq, Hk, scale, impl="mma")  # noqa: E731
    ws = torch.empty(o.flash_attn_bwd_ws_numel(B, T, Hk), device=dev)
    bwd = lambda: o.flash_attn_bwd(q, k, v, out, dout, lse, delta, dqkv[:, : Hq * D],  # noqa: E731
                                   dqkv[:, Hq * D:(Hq + Hk) * D], dqkv[:, (Hq + Hk) * D:], B, T, Hq, Hk, scale,
                                   impl="tc", ws=ws)
    bwd_mma = lambda: o.flash_attn_bwd(q, k, v, out, dout, lse, delta, dqkv[:, : Hq * D],  # noqa: E731
                                       dqkv[:, Hq * D:(Hq + Hk) * D], dqkv[:, (Hq + Hk) * D:], B, T, Hq, Hk, scale,
                                       impl="mma")
    t_fm = timed(fwd_mma, steps)
    fwd()
    t_bm = timed(bwd_mma, steps)
    t_f, t_b = timed(fwd, steps), timed(bwd, steps)
    # PyTorch SDPA on [B, H, T, D] views (GQA by repeating K/V heads)
    qt = q.reshape(B, T, Hq, D).transpose(1, 2).contiguous()
    kt = k.reshape(B, T, Hk, D).transpose(1, 2).repeat_interleave(Hq // Hk, 1).contiguous()
    vt = v.reshape(B, T, Hk, D).transpose(1, 2).repeat_interleave(Hq // Hk, 1).contiguous()
    t_sdpa = timed(lambda: F.scaled_dot_product_attention(qt, kt, vt, is_causal=True), steps)
    qg, kg, vg = (t.detach().requires_grad_() for t in (qt, kt, vt))
    og = F.scaled_dot_product_attention(qg, kg, vg, is_causal=True)
    gt = torch.randn_like(og)
    t_sdpa_b = timed(lambda: torch.autograd.grad(og, (qg, kg, vg), gt, retain_graph=True), steps)
    err = (out.float().view(B, T, Hq, D).transpose(1, 2) -
           F.scaled_dot_product_attention(qt, kt, vt, is_causal=True).float()).abs().max().item()
    fl = 2.0 * B * Hq * T * T * D
    ref = bench_reference(qt, kt, vt, ref_steps) if ref_steps > 0 else None
    r = {"shape": name, "B": B, "T": T, "Hq": Hq, "Hk": Hk, "D": D,
         "fwd_ms": t_f, "fwd_tflops": fl / t_f / 1e9, "fwd_mma_sync_ms": t_fm, "bwd_mma_sync_ms": t_bm, "bwd_ms": t_b, "bwd_tflops": 2.5 * fl / t_b / 1e9,
         "sdpa_fwd_ms": t_sdpa, "sdpa_bwd_ms": t_sdpa_b, "max_abs_diff_vs_sdpa": err}
    print(f"{name:22s} fwd {t_f * 1e3:8.1f} us {r['fwd_tflops']:6.0f} TF/s (mma.sync {t_fm * 1e3:.1f} us) | bwd {t_b * 1e3:8.1f} us "
          f"{r['bwd_tflops']:6.0f} TF/s (mma.sync {t_bm * 1e3:.1f} us) | torch SDPA fwd {t_sdpa * 1e3:8.1f} us bwd {t_sdpa_b * 1e3:8.1f} us "
          f"| max|diff| {err:.3g}")
    if ref is not None:
        r.update({"reference_fwd_ms": ref[0], "reference_fwd_tflops_full": 2 * fl / ref[0] / 1e9,
                  "reference_max_abs_diff_vs_sdpa_fp32": ref[1], "fwd_speedup_vs_reference": ref[0] / t_f})
        print(f"{'':22s} reference kernel (fp32, non-causal) fwd {ref[0] * 1e3:10.1f} us "
              f"{r['reference_fwd_tflops_full']:6.2f} TF/s of full work | max|diff| vs fp32 SDPA {ref[1]:.3g} "
              f"| this framework's tcgen05 fwd is {ref[0] / t_f:.0f}x faster")
    return r


def main():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--ref-steps", type=int, default=3, help="timed calls of the reference kernel (0: skip it)")
    a = p.parse_args()
    if not torch.cuda.is_available():
        print(json.dumps({"benchmark": "attention", "skipped": "no CUDA device"}))
        return
    res = [bench_shape(n, *s, a.steps, a.ref_steps) for n, s in SHAPES.items()]
    print(json.dumps({"benchmark": "attention", "timing": "CUDA events, mean after 3 warm-ups", "results": res}))


if __name__ == "__main__":
    main()
