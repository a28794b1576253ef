"""Host-side failure detection and restart (turbol_b200.launch), on CPU with
gloo ranks: a rank that exits non-zero, and a rank that goes silent (no
heartbeat), both end the attempt; the relaunch resumes from the per-rank
checkpoint and finishes with the same result as an uninterrupted run."""
import os
import random
import socket
import sys

import pytest

from turbol_b200.launch import main as launch_main

HERE = os.path.dirname(os.path.abspath(__file__))
WORKER = os.path.join(HERE, "launch_worker.py")


_RNG = random.Random()


def _port(span: int = 2):
    """A port p with p .. p + span - 1 all free (the launcher relaunches on
    port + attempt), taken below the kernel's ephemeral range: a port the
    kernel handed out (bind to 0) can be followed by one that the first
    attempt's own gloo connections are using."""
    rng = _RNG
    lo = 20000
    try:
        with open("/proc/sys/net/ipv4/ip_local_port_range") as f:
            lo = min(lo, int(f.read().split()[0]) - 2000)
    except (OSError, ValueError, IndexError):
        pass
    for _ in range(200):
        p = rng.randrange(max(1024, lo - 8000), lo)
        socks = []
        try:
            for q in range(p, p + span):
                s = socket.socket()
                socks.append(s)
                s.bind(("127.0.0.1", q))
            return p
        except OSError:
            continue
        finally:
            for s in socks:
                s.close()
    raise RuntimeError("no free port pair")


def _results(d, world):
    out = []
    for r in range(world):
        with open(os.path.join(d, f"done{r}.txt")) as f:
            step, acc, attempt = f.read().split()
            out.append((int(step), float(acc), int(attempt)))
    return out


@pytest.mark.parametrize("mode", ["ok", "crash", "hang"])
def test_restart_resumes_from_checkpoint(tmp_path, mode):
    world, steps = 2, 5
    argv = ["--nproc", str(world), "--max-restarts", "1", "--port", str(_port()),
            "--heartbeat-timeout", "6", WORKER, mode, str(tmp_path), str(steps)]
    assert launch_main(argv) == 0
    res = _results(tmp_path, world)
    # sum over ranks of (rank + 1) = 3, accumulated once per step
    assert all(step == steps and acc == 3.0 * steps for step, acc, _ in res)
    assert all(att == (0 if mode == "ok" else 1) for _, _, att in res)


def test_gives_up_after_max_restarts(tmp_path):
    bad = tmp_path / "bad.py"
    bad.write_text("import sys; sys.exit(int(__import__('os').environ['RANK']) + 1)\n")
    argv = ["--nproc", "2", "--max-restarts", "1", "--port", str(_port()), str(bad)]
    assert launch_main(argv) == 1
