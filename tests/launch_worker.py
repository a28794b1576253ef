"""Worker for test_launch.py: a gloo training loop that checkpoints its step
counter and, on demand, fails on the first attempt (exits non-zero, or stops
beating its heartbeat) so the launcher has to restart it."""
import datetime
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from turbol_b200.launch import heartbeat  # noqa: E402


def main():
    mode, ckpt_dir, steps = sys.argv[1], sys.argv[2], int(sys.argv[3])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    attempt = int(os.environ["TURBOL_RESTART"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
    path = os.path.join(ckpt_dir, f"rank{rank}.pt")
    state = torch.load(path) if os.path.exists(path) else {"step": 0, "acc": torch.zeros(4)}
    for step in range(state["step"], steps):
        heartbeat()
        if attempt == 0 and rank == 1 and step == 2:
            if mode == "crash":
                sys.exit(3)
            if mode == "hang":  # host-side silence: sleeps, never reaches the next collective
                time.sleep(120)
        x = torch.full((4,), float(rank + 1))
        dist.all_reduce(x)
        state["acc"] += x
        state["step"] = step + 1
        torch.save(state, path)
    with open(os.path.join(ckpt_dir, f"done{rank}.txt"), "w") as f:
        f.write(f"{state['step']} {float(state['acc'][0])} {attempt}\n")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
