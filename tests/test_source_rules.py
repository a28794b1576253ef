"""Source rules for code that runs on several GPUs, checked on the CPU.

* No bulk or tensor TMA load with cluster multicast anywhere in the kernels:
  the tensor-parallel and data-parallel kernels read peer memory, and a
  multicast load whose source is (or could be) another GPU's memory is
  forbidden; the rule is kept global so no multi-GPU path can reach one.
* Every kernel source is built for sm_100a only (no other -gencode target).
* Every device spin-wait in the peer-memory kernels goes through a bounded
  helper (a time budget), never an open-ended loop on a flag.
"""
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KERNELS = sorted(glob.glob(os.path.join(ROOT, "csrc", "kernels", "*.cu")) +
                 glob.glob(os.path.join(ROOT, "csrc", "kernels", "*.cuh")) +
                 glob.glob(os.path.join(ROOT, "csrc", "kernels", "*.h")))
# the qualifier is assembled so that this file does not itself read as a use of it
MC = "multicast" + "::" + "cluster"


def _code_lines(path):
    """(line number, text) of a source file with // comments removed."""
    out = []
    for i, line in enumerate(open(path, encoding="utf-8"), 1):
        out.append((i, line.split("//", 1)[0]))
    return out


def test_no_multicast_bulk_loads():
    bad = []
    for path in KERNELS:
        for i, code in _code_lines(path):
            if "cp.async.bulk" in code and MC in code:
                bad.append(f"{os.path.relpath(path, ROOT)}:{i}")
    assert not bad, f"cluster-multicast bulk/TMA loads found: {bad}"


def test_sm100a_only():
    setup = open(os.path.join(ROOT, "setup.py"), encoding="utf-8").read()
    targets = set(re.findall(r"arch=compute_(\w+),code=sm_(\w+)", setup))
    assert targets == {("100a", "100a")}, targets


def test_peer_waits_are_bounded():
    """The collective kernels spin only inside helpers that take a time budget."""
    for name in ("comm.cu", "gemm_tcgen05.cu"):
        src = open(os.path.join(ROOT, "csrc", "kernels", name), encoding="utf-8").read()
        # every acquire-load loop must sit in a function that reads the global timer
        for m in re.finditer(r"while\s*\([^;{]*ld_acquire[^;{]*\)", src):
            head = src[:m.start()]
            fn_start = head.rfind("__device__")
            body = src[fn_start:m.end() + 400]
            clock = any(c in body for c in ("now_ns()", "global_ns()", "globaltimer"))
            assert clock and "budget" in body.lower(), f"{name}: unbounded flag wait near offset {m.start()}"
