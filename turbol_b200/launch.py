"""Process launcher with failure detection and restart.

    python -m turbol_b200.launch --nproc 8 [--max-restarts 2] [--port 29500] script.py [args...]

Starts one worker process per rank with the torchrun environment (RANK,
LOCAL_RANK, WORLD_SIZE, MASTER_ADDR=127.0.0.1, MASTER_PORT) plus
TURBOL_RESTART (the attempt number), and watches them:

* a worker that exits non-zero, or that stops updating its heartbeat file for
  ``--heartbeat-timeout`` seconds (when the worker calls
  :func:`heartbeat`), marks the attempt failed;
* the other workers of a failed attempt are stopped (SIGTERM, then SIGKILL
  after a grace period) by their exact process ids;
* the attempt is relaunched, up to ``--max-restarts`` times, on a new port;
  workers resume from their last checkpoint (``turbol_b200.load_checkpoint``),
  which is how training survives a failed rank.

Failure detection is entirely on the host: a dead or silent rank is noticed by
its exit status or its heartbeat, never by a device-side fault.
"""
from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
import tempfile
import time
from typing import List, Optional


def heartbeat():
    """Called by a worker (e.g. once per training step) to prove it is alive."""
    path = os.environ.get("TURBOL_HEARTBEAT")
    if path:
        with open(path, "w") as f:
            f.write(f"{time.time()}\n")


def _stop(procs: List[subprocess.Popen], grace: float = 10.0):
    for p in procs:
        if p.poll() is None:
            p.send_signal(signal.SIGTERM)
    t0 = time.time()
    for p in procs:
        while p.poll() is None and time.time() - t0 < grace:
            time.sleep(0.05)
        if p.poll() is None:
            p.kill()
            p.wait()


def run_attempt(cmd: List[str], nproc: int, port: int, attempt: int, hb_dir: str, hb_timeout: Optional[float],
                env_extra=None) -> int:
    """Runs one attempt; returns 0 when every worker exited 0."""
    procs, beats = [], []
    for r in range(nproc):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(nproc), LOCAL_WORLD_SIZE=str(nproc),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), TURBOL_RESTART=str(attempt))
        hb = os.path.join(hb_dir, f"hb_{attempt}_{r}")
        env["TURBOL_HEARTBEAT"] = hb
        if env_extra:
            env.update(env_extra)
        beats.append(hb)
        procs.append(subprocess.Popen(cmd, env=env))
    start = time.time()
    status = 0
    while True:
        codes = [p.poll() for p in procs]
        if any(c not in (None, 0) for c in codes):
            bad = [r for r, c in enumerate(codes) if c not in (None, 0)]
            print(f"[turbol.launch] attempt {attempt}: rank(s) {bad} exited with {[codes[r] for r in bad]}",
                  flush=True)
            status = 1
            break
        if all(c == 0 for c in codes):
            break
        if hb_timeout is not None:
            now = time.time()
            for r, hb in enumerate(beats):
                if codes[r] is not None:
                    continue
                last = os.path.getmtime(hb) if os.path.exists(hb) else start
                if now - last > hb_timeout:
                    print(f"[turbol.launch] attempt {attempt}: rank {r} silent for {now - last:.1f} s", flush=True)
                    status = 2
            if status:
                break
        time.sleep(0.1)
    if status:
        _stop(procs)
    return status


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--nproc", type=int, default=1)
    ap.add_argument("--max-restarts", type=int, default=0)
    ap.add_argument("--port", type=int, default=29500)
    ap.add_argument("--heartbeat-timeout", type=float, default=None)
    ap.add_argument("script")
    ap.add_argument("args", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cmd = [sys.executable, a.script] + a.args
    with tempfile.TemporaryDirectory(prefix="turbol_launch_") as hb_dir:
        for attempt in range(a.max_restarts + 1):
            rc = run_attempt(cmd, a.nproc, a.port + attempt, attempt, hb_dir, a.heartbeat_timeout)
            if rc == 0:
                return 0
            if attempt < a.max_restarts:
                print(f"[turbol.launch] restarting (attempt {attempt + 1} of {a.max_restarts})", flush=True)
    print("[turbol.launch] giving up", flush=True)
    return 1


if __name__ == "__main__":
    sys.exit(main())
