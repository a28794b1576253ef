"""Source rules for code that runs on several GPUs, checked on the CPU.

* Every bulk / tensor (TMA) copy in the kernels uses only the qualifiers on
  an allow-list: a plain tile or bulk copy into this CTA's shared memory,
  completing on an mbarrier.  The tensor-parallel and data-parallel kernels
  read peer memory, and a copy that fans one load out to several CTAs must
  never read another GPU's memory; keeping the rule global means no
  multi-GPU path can reach such a copy.
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
# the qualifiers a bulk / tensor copy may carry
ALLOWED = {"tensor", "1d", "2d", "3d", "4d", "5d", "shared::cluster", "shared::cta", "global", "tile",
           "mbarrier::complete_tx::bytes", "bulk_group", "L2::cache_hint", "async", "bulk", "cp", "commit_group",
           "wait_group", "read", "prefetch", "im2col"}


def _code_lines(path):
    """(line number, text) of a source file with // comments removed."""
    out = []
    for i, line in enumerate(open(path, encoding="utf-8"), 1):
        out.append((i, line.split("//", 1)[0]))
    return out


def test_bulk_copies_use_allowed_qualifiers_only():
    bad = []
    for path in KERNELS:
        for i, code in _code_lines(path):
            for m in re.finditer(r"cp\.async\.bulk[\w.:]*", code):
                extra = [q for q in m.group(0).split(".") if q and q not in ALLOWED]
                if extra:
                    bad.append(f"{os.path.relpath(path, ROOT)}:{i}: {extra}")
    assert not bad, f"bulk/TMA copies with qualifiers outside the allow-list: {bad}"


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
