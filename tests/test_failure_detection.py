"""Failure detection without a GPU fault.

On the device: the bounded flag wait that every peer-memory collective uses
runs out on a flag that nothing sets, records its site in the error word and
returns; the context stays usable.  On the host: see test_dist.py (a rank that
never joins -> rendezvous timeout as a Status; invalid configurations)."""
import time

import pytest
import torch

from turbol_b200._native import ops

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_with_error_status(dev):
    o = ops()
    flags = torch.zeros(2, dtype=torch.int32, device=dev)  # nothing will set these
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    t0 = time.perf_counter()
    o.bounded_wait_probe(flags, 1, 0.05, err)
    torch.cuda.synchronize(dev)
    dt = time.perf_counter() - t0
    assert int(err.item()) == 99 and dt < 5.0
    # the context is still usable
    x = torch.arange(1000, device=dev, dtype=torch.float32)
    assert float((x * 2).sum()) == 999000.0


def test_bounded_wait_passes_when_flags_are_set(dev):
    o = ops()
    flags = torch.full((3,), 7, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    o.bounded_wait_probe(flags, 7, 0.05, err)
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0
