#!/usr/bin/env python
"""Checkpoint save / load time for a trainer state of a given size.

    python benchmarks/bench_checkpoint.py [--params 100000000] [--device cpu|cuda] [--dir PATH]

The state mirrors what the trainers save per rank: the fp32 flat weights
("policy"), the Adam moments m and v ("optim", 2 x the weights) and a small
trainer record.  Times: the blocking save (device -> host snapshot + write +
completion marker), the time a background save blocks the caller (the host
snapshot only), and the load.  Reported as seconds and GB/s of state.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import tempfile
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from turbol_b200.utils.checkpoint import load_checkpoint, save_checkpoint  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--params", type=int, default=100_000_000)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--dir", default=None, help="target directory (default: a temporary one)")
    ap.add_argument("--reps", type=int, default=2)
    a = ap.parse_args()
    dev = torch.device(a.device)
    n = a.params
    flat = torch.randn(n, device=dev)
    state = {"policy": {"flat": flat}, "optim": {"m": torch.randn(n, device=dev), "v": torch.rand(n, device=dev),
                                                 "step": torch.tensor(7)},
             "iteration": 3, "rng": torch.get_rng_state()}
    nbytes = 3 * n * 4
    root = a.dir or tempfile.mkdtemp(prefix="turbol_ckpt_bench_")
    res = {"benchmark": "checkpoint", "params": n, "state_bytes": nbytes, "device": str(dev), "dir": root}
    try:
        save_s, snap_s, load_s = [], [], []
        for r in range(a.reps):
            t0 = time.perf_counter()
            save_checkpoint(root, 2 * r + 1, state=state, write_config=False, background=False)
            save_s.append(time.perf_counter() - t0)
            t0 = time.perf_counter()
            h = save_checkpoint(root, 2 * r + 2, state=state, write_config=False, background=True)
            snap_s.append(time.perf_counter() - t0)
            h.wait()
            t0 = time.perf_counter()
            st = load_checkpoint(root, step=2 * r + 2)
            load_s.append(time.perf_counter() - t0)
            assert torch.equal(st["policy"]["flat"], flat.cpu())
        res.update({"save_s": min(save_s), "save_gb_s": nbytes / min(save_s) / 1e9,
                    "background_blocks_s": min(snap_s), "load_s": min(load_s), "load_gb_s": nbytes / min(load_s) / 1e9})
    finally:
        if a.dir is None:
            shutil.rmtree(root, ignore_errors=True)
    print(json.dumps(res))


if __name__ == "__main__":
    main()
