"""GAE and GRPO advantage kernels vs the fp32 PyTorch oracle."""
import pytest
import torch

from turbol_b200.ops import reference as ref
from turbol_b200.ops.rl import gae, grpo_advantage


def test_gae_reference_hand_case():
    r = torch.tensor([[1.0], [1.0], [1.0]])
    v = torch.tensor([[0.5], [0.5], [0.5], [2.0]])
    d = torch.tensor([[0], [1], [0]], dtype=torch.uint8)
    adv, ret = ref.gae(r, v, d, gamma=0.9, lam=0.8)
    # t=2: delta = 1 + .9*2 - .5 = 2.3 ; t=1 done: delta = 1 - .5 = .5, A=.5 ; t=0: delta=1+.45-.5=.95, A=.95+.72*.5
    assert torch.allclose(adv[:, 0], torch.tensor([0.95 + 0.72 * 0.5, 0.5, 2.3]))
    assert torch.allclose(ret, adv + v[:3])


def test_grpo_advantage_cpu():
    r = torch.tensor([1.0, 2.0, 3.0, 4.0, 0.0, 0.0, 0.0, 0.0])
    a = grpo_advantage(r, 4)
    assert torch.allclose(a[:4], (r[:4] - 2.5) / (r[:4].std() + 1e-4))
    assert torch.all(a[4:] == 0)


@pytest.mark.gpu
@pytest.mark.parametrize("T,N", [(1, 7), (17, 33), (64, 1000), (256, 4096), (128, 65536), (3, 40000)])
def test_gae_kernel_matches_oracle(T, N, dev):
    g = torch.Generator().manual_seed(T * 1000 + N)
    r = torch.rand(T, N, generator=g) * 2 - 1
    v = torch.randn(T + 1, N, generator=g)
    d = (torch.rand(T, N, generator=g) < 0.05).to(torch.uint8)
    d[0, :3] = 1
    d[-1, 3:6] = 1
    ea, er = ref.gae(r.double(), v.double(), d, 0.99, 0.95)
    stats = torch.zeros(2, dtype=torch.float64, device=dev)
    a, rt = gae(r.to(dev), v.to(dev), d.to(dev), 0.99, 0.95, stats=stats)
    assert torch.allclose(a.cpu().double(), ea, atol=2e-4, rtol=1e-4)
    assert torch.allclose(rt.cpu().double(), er, atol=2e-4, rtol=1e-4)
    s = stats.cpu()
    assert abs(float(s[0]) - float(ea.sum())) < 1e-3 * max(1.0, float(ea.abs().sum()))
    assert abs(float(s[1]) - float((ea ** 2).sum())) < 1e-3 * max(1.0, float((ea ** 2).sum()))


@pytest.mark.gpu
def test_gae_bool_dones(dev):
    T, N = 40, 300
    r = torch.rand(T, N, device=dev)
    v = torch.rand(T + 1, N, device=dev)
    d = torch.rand(T, N, device=dev) < 0.1
    a, _ = gae(r, v, d)
    ea, _ = ref.gae(r.cpu(), v.cpu(), d.cpu())
    assert torch.allclose(a.cpu(), ea, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("G", [1, 2, 8, 16])
def test_grpo_kernel(G, dev):
    r = torch.rand(64 * G, generator=torch.Generator().manual_seed(G))
    got = grpo_advantage(r.to(dev), G).cpu()
    exp = ref.grpo_advantage(r, G)
    assert torch.allclose(got, exp, atol=1e-5)


@pytest.mark.parametrize("T,N", [(1, 5), (37, 130), (256, 4096)])
def test_gae_host_sweep_matches_oracle(T, N):
    """CPU tensors take the core's one-sweep GAE; it equals the float64 oracle
    and accumulates the advantage sum and sum of squares."""
    g = torch.Generator().manual_seed(T)
    r = torch.randn(T, N, generator=g)
    v = torch.randn(T + 1, N, generator=g)
    d = torch.rand(T, N, generator=g) < 0.05
    stats = torch.zeros(2, dtype=torch.float64)
    a, rt = gae(r, v, d, 0.99, 0.95, stats=stats)
    ea, er = ref.gae(r.double(), v.double(), d, 0.99, 0.95)
    assert torch.allclose(a.double(), ea, atol=1e-4, rtol=1e-4)
    assert torch.allclose(rt.double(), er, atol=1e-4, rtol=1e-4)
    assert abs(float(stats[0]) - float(ea.sum())) < 1e-3 * max(1.0, float(ea.abs().sum()))
    assert abs(float(stats[1]) - float((ea * ea).sum())) < 1e-3 * max(1.0, float((ea * ea).sum()))


def test_gae_host_split_over_threads_matches_one_thread():
    """A [128, 40000] sweep is split by environment blocks over 4 threads:
    advantages and returns are bit-identical to one thread's (each
    environment's recurrence is the same), the statistics agree to rounding,
    and both equal the float64 oracle."""
    g = torch.Generator().manual_seed(9)
    T, N = 128, 40000
    r = torch.randn(T, N, generator=g)
    v = torch.randn(T + 1, N, generator=g)
    d = torch.rand(T, N, generator=g) < 0.05
    out = []
    prev = torch.get_num_threads()
    try:
        for threads in (1, 4):
            torch.set_num_threads(threads)
            stats = torch.zeros(2, dtype=torch.float64)
            a, rt = gae(r, v, d, 0.99, 0.95, stats=stats)
            out.append((a, rt, stats))
    finally:
        torch.set_num_threads(prev)
    assert torch.equal(out[0][0], out[1][0]) and torch.equal(out[0][1], out[1][1])
    assert torch.allclose(out[0][2], out[1][2], rtol=1e-9, atol=1e-6)
    ea, _ = ref.gae(r.double(), v.double(), d, 0.99, 0.95)
    assert torch.allclose(out[1][0].double(), ea, atol=1e-4, rtol=1e-4)


def test_static_scratch_gae_bound_cpu():
    """The allocation-free GAE entry point's size check (host arithmetic, no
    GPU): fits() agrees with the 1 MiB array for every shape probed, and under
    the chunk rule no shape needs more than 196,608 floats, so the rejection
    branch only guards a future change of that rule."""
    import ctypes

    import turbol_b200
    from turbol_b200._native import ops

    lib = ctypes.CDLL(turbol_b200.turbol_core.__file__)
    fits = lib.tb_gae_static_scratch_fits
    fits.restype, fits.argtypes = ctypes.c_int, [ctypes.c_int, ctypes.c_int]
    worst = 0
    for N in list(range(1, 300)) + [511, 513, 1000, 4095, 4097, 16383, 32767, 32768, 65536]:
        for T in (1, 2, 7, 64, 65, 256, 4096):
            need = ops().gae_scratch_numel(T, N)
            worst = max(worst, need)
            assert fits(T, N) == (1 if need <= 256 * 1024 else 0), (T, N, need)
    assert worst < 196608, worst
