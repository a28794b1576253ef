"""The allocation-free GAE entry point (tb_gae_static_scratch), called through
its exported C symbol the way a caller that cannot allocate device memory
would: it hands over raw device pointers and a stream, and the library uses
its compiled-in workspace.  Its output must match the regular entry point
(ops.gae, which takes a caller-allocated workspace) on two calls in a row.

This file sorts last so that a run stopping at the first failure has already
run every other test."""
import ctypes

import pytest
import torch

import turbol_b200
from turbol_b200._native import ops

pytestmark = pytest.mark.gpu


def _lib():
    lib = ctypes.CDLL(turbol_b200.turbol_core.__file__)
    fn = lib.tb_gae_static_scratch
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                           ctypes.c_void_p]
    fits = lib.tb_gae_static_scratch_fits
    fits.restype = ctypes.c_int
    fits.argtypes = [ctypes.c_int, ctypes.c_int]
    return fn, fits


@pytest.mark.parametrize("T,N", [(64, 1000), (256, 4096), (37, 513)])
def test_static_scratch_gae_matches_regular_entry_point(T, N):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fn, fits = _lib()
    assert fits(T, N) == 1
    g = torch.Generator().manual_seed(T + N)
    stream = torch.cuda.current_stream(dev)
    for call in range(2):  # two calls in a row share (and reuse) the workspace
        r = (torch.rand(T, N, generator=g) * 2 - 1).to(dev)
        v = torch.randn(T + 1, N, generator=g).to(dev)
        d = (torch.rand(T, N, generator=g) < 0.05).to(torch.uint8).to(dev)
        adv_ref, ret_ref = torch.empty(T, N, device=dev), torch.empty(T, N, device=dev)
        st_ref = torch.zeros(2, dtype=torch.float64, device=dev)
        ops().gae(r, v, d, adv_ref, ret_ref, st_ref, None, 0.99, 0.95)
        adv, ret = torch.empty(T, N, device=dev), torch.empty(T, N, device=dev)
        st = torch.zeros(2, dtype=torch.float64, device=dev)
        err = fn(r.data_ptr(), v.data_ptr(), d.data_ptr(), adv.data_ptr(), ret.data_ptr(), st.data_ptr(), T, N,
                 0.99, 0.95, stream.cuda_stream)
        assert err == 0, f"call {call}: cudaError {err}"
        torch.cuda.synchronize(dev)
        assert torch.allclose(adv, adv_ref, atol=1e-5, rtol=1e-5), call
        assert torch.allclose(ret, ret_ref, atol=1e-5, rtol=1e-5), call
        assert torch.allclose(st, st_ref, rtol=1e-9, atol=1e-6), call


def test_static_scratch_size_bound():
    # fits() is exactly "the chunked scan's workspace is within the 1 MiB array"
    # (262,144 floats); with the chunk-count rule every shape in this range fits
    _, fits = _lib()
    for T, N in [(1, 7), (2, 16384), (64, 4100), (256, 1000), (4096, 30000), (128, 65536), (3000, 33)]:
        need = ops().gae_scratch_numel(T, N)
        assert fits(T, N) == (1 if need <= 256 * 1024 else 0), (T, N, need)
