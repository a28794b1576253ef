"""RingBuffer and PrioritizedReplayBuffer: the reference's RingBufferTest cases
(turbol_vllm/tests/test_ring_buffer.cpp, turbol/tests/test_ring_buffer.cpp:46-83)
plus statistical checks of the samplers and kernel-vs-CPU equality."""
import numpy as np
import pytest
import torch

import turbol_b200 as turbol


def _t(x):
    return turbol.from_torch(torch.as_tensor(x))


def test_push_sample_shapes():
    b = turbol.RingBuffer(capacity=16, obs_dim=4, act_dim=2, device="cpu")
    assert b.size() == 0 and b.capacity() == 16
    for i in range(5):
        assert b.push(_t(torch.full((4,), float(i))), _t(torch.zeros(2)), _t(torch.ones(1)), False).ok()
    assert b.size() == 5
    o, a, r, d = turbol.Tensor(), turbol.Tensor(), turbol.Tensor(), turbol.Tensor()
    assert b.sample(8, o, a, r, d).ok()
    assert o.shape().to_list() == [8, 4] and a.shape().to_list() == [8, 2]
    assert r.shape().to_list() == [8] and d.dtype() == "bool"
    b.clear()
    assert b.size() == 0


def test_sample_rejects_empty_buffer():
    b = turbol.RingBuffer(capacity=4, obs_dim=2, act_dim=1, device="cpu")
    o, a, r, d = turbol.Tensor(), turbol.Tensor(), turbol.Tensor(), turbol.Tensor()
    assert not b.sample(2, o, a, r, d).ok()


def test_wraparound_keeps_newest_and_rows_consistent():
    b = turbol.RingBuffer(capacity=4, obs_dim=3, act_dim=2, device="cpu")
    for i in range(6):
        b.push(_t(torch.full((3,), float(i))), _t(torch.full((2,), float(10 * i))), _t(torch.tensor([float(i)])),
               i % 2 == 1)
    assert b.size() == 4
    o, a, r, d = b.sample_batch(200)
    vals = set(o[:, 0].tolist())
    assert vals <= {2.0, 3.0, 4.0, 5.0} and len(vals) == 4
    assert torch.all(o[:, 0] == o[:, 2]) and torch.all(a[:, 0] == 10 * o[:, 0]) and torch.all(r == o[:, 0])
    assert torch.all(d == (o[:, 0].long() % 2 == 1))


def test_push_batch_larger_than_capacity():
    b = turbol.RingBuffer(capacity=8, obs_dim=1, act_dim=1, device="cpu")
    x = torch.arange(20, dtype=torch.float32)
    b.push_batch(_t(x[:, None]), _t(x[:, None]), _t(x), _t(torch.zeros(20, dtype=torch.bool)))
    o, *_ = b.storage()
    assert sorted(o[:, 0].tolist()) == list(range(12, 20))


def test_host_sample_indices_follow_the_philox_stream():
    """Index i of sample call k is Philox(seed; i, k, 0, 0x52504C59) word 0,
    reduced to [0, size) by multiply-shift (the device kernel's definition);
    batch sizes that are not multiples of the host's 8-lane batches."""
    from turbol_b200.ops import reference as ref

    cap = 1000
    b = turbol.RingBuffer(cap, 3, 1, "cpu", seed=77)
    b.push_batch(_t(torch.randn(cap, 3)), _t(torch.randn(cap, 1)), _t(torch.randn(cap)),
                 _t(torch.zeros(cap, dtype=torch.bool)))
    for k, n in enumerate((37, 8, 1, 100)):
        got = b.sample_indices(n).tolist()
        exp = [(ref.philox4x32_10(77, i, k, 0, 0x52504C59)[0] * cap) >> 32 for i in range(n)]
        assert got == exp, k


def test_host_sample_equals_indices_then_gather():
    """On the CPU, sample() draws the same indices as sample_indices() (same
    counter stream) and returns the rows gather() returns for them."""
    cap = 500
    b1 = turbol.RingBuffer(cap, 5, 2, "cpu", seed=9)
    b2 = turbol.RingBuffer(cap, 5, 2, "cpu", seed=9)
    g = torch.Generator().manual_seed(2)
    o, a, r = torch.randn(cap, 5, generator=g), torch.randn(cap, 2, generator=g), torch.randn(cap, generator=g)
    d = torch.rand(cap, generator=g) < 0.3
    for b in (b1, b2):
        b.push_batch(_t(o), _t(a), _t(r), _t(d))
    for n in (13, 64):
        so, sa, sr, sd = turbol.Tensor(), turbol.Tensor(), turbol.Tensor(), turbol.Tensor()
        assert b1.sample(n, so, sa, sr, sd).ok()
        exp = b2.gather(b2.sample_indices(n))
        for x, y in zip((so, sa, sr, sd), exp):
            assert torch.equal(x.torch(), y)


def test_uniform_sampling_chi_square():
    cap = 64
    b = turbol.RingBuffer(capacity=cap, obs_dim=1, act_dim=1, device="cpu", seed=7)
    x = torch.arange(cap, dtype=torch.float32)
    b.push_batch(_t(x[:, None]), _t(x[:, None]), _t(x), _t(torch.zeros(cap, dtype=torch.bool)))
    idx = torch.cat([b.sample_indices(4096) for _ in range(16)]).long()
    counts = torch.bincount(idx, minlength=cap).double()
    exp = idx.numel() / cap
    chi2 = float(((counts - exp) ** 2 / exp).sum())
    assert chi2 < 63 + 4 * (2 * 63) ** 0.5  # mean 63, sd ~11.2


def test_per_proportional_and_weights():
    cap = 32
    b = turbol.PrioritizedReplayBuffer(capacity=cap, obs_dim=1, act_dim=1, alpha=0.6, beta=0.4, device="cpu", seed=3)
    x = torch.arange(cap, dtype=torch.float32)
    b.push_batch(_t(x[:, None]), _t(x[:, None]), _t(x), _t(torch.zeros(cap, dtype=torch.bool)))
    pr = torch.rand(cap, generator=torch.Generator().manual_seed(0)) + 0.05
    b.update_priorities(torch.arange(cap), pr)
    p = pr.double() ** 0.6
    p = p / p.sum()
    assert abs(b.total_priority() - float((pr.double() ** 0.6).sum())) < 1e-3
    counts = torch.zeros(cap, dtype=torch.float64)
    for _ in range(64):
        o, a, r, d, idx, w = b.sample_prioritized(256)
        counts += torch.bincount(idx, minlength=cap).double()
        assert torch.all(o[:, 0].long() == idx)
        # IS weights: (N P(i))^-beta normalized by the batch max
        wi = (cap * p[idx]) ** -0.4
        assert torch.allclose(w.double(), wi / wi.max(), atol=1e-4)
    freq = counts / counts.sum()
    assert torch.allclose(freq, p, atol=0.01)


@pytest.mark.gpu
def test_gpu_push_gather_matches_cpu(dev):
    cap, od, ad = 1000, 7, 3  # odd row sizes: 4-byte path
    rng = torch.Generator().manual_seed(0)
    bc = turbol.RingBuffer(cap, od, ad, "cpu")
    bg = turbol.RingBuffer(cap, od, ad, dev)
    for B in (300, 450, 700):  # wraps
        o = torch.randn(B, od, generator=rng)
        a = torch.randn(B, ad, generator=rng)
        r = torch.randn(B, generator=rng)
        d = torch.rand(B, generator=rng) < 0.1
        for buf, dv in ((bc, "cpu"), (bg, dev)):
            assert buf.push_batch(_t(o.to(dv)), _t(a.to(dv)), _t(r.to(dv)), _t(d.to(dv))).ok()
    assert bc.size() == bg.size() == cap and bc.head() == bg.head()
    for x, y in zip(bc.storage(), bg.storage()):
        assert torch.equal(x, y.cpu())
    idx = torch.randint(0, cap, (5000,), generator=rng, dtype=torch.int32)
    for x, y in zip(bc.gather(idx), bg.gather(idx.to(dev))):
        assert torch.equal(x, y.cpu())


@pytest.mark.gpu
def test_gpu_vectorized_rows_and_sampling(dev):
    cap, od, ad = 1 << 16, 64, 8  # 256-byte and 32-byte rows: 16-byte vector path
    b = turbol.RingBuffer(cap, od, ad, dev, seed=5)
    o = torch.randn(cap, od, device=dev)
    a = torch.randn(cap, ad, device=dev)
    r = torch.rand(cap, device=dev) * 2 - 1
    d = torch.rand(cap, device=dev) < 0.01
    b.push_batch(_t(o), _t(a), _t(r), _t(d))
    idx = b.sample_indices(65536)
    assert idx.is_cuda and int(idx.min()) >= 0 and int(idx.max()) < cap
    so, sa, sr, sd = b.gather(idx)
    il = idx.long()
    assert torch.equal(so, o[il]) and torch.equal(sa, a[il]) and torch.equal(sr, r[il]) and torch.equal(sd, d[il])
    counts = torch.bincount(torch.cat([b.sample_indices(65536) for _ in range(8)]).long() % 64, minlength=64)
    exp = 8 * 65536 / 64
    assert float(((counts.double() - exp) ** 2 / exp).sum()) < 63 + 5 * (2 * 63) ** 0.5


@pytest.mark.gpu
def test_gpu_per_matches_cpu_and_distribution(dev):
    cap = 5000
    rng = torch.Generator().manual_seed(2)
    pr = torch.rand(cap, generator=rng) + 0.01
    bufs = []
    for dv in ("cpu", dev):
        b = turbol.PrioritizedReplayBuffer(cap, 2, 1, alpha=0.6, beta=0.4, device=dv, seed=9)
        x = torch.arange(cap, dtype=torch.float32)
        b.push_batch(_t(torch.stack([x, x], 1).to(dv)), _t(x[:, None].to(dv)), _t(x.to(dv)),
                     _t(torch.zeros(cap, dtype=torch.bool, device=dv)))
        b.update_priorities(torch.arange(cap, device=dv), pr.to(dv))
        bufs.append(b)
    tc, tg = bufs[0].tree(), bufs[1].tree().cpu()
    assert torch.allclose(tc, tg, rtol=1e-4, atol=1e-4)
    counts = torch.zeros(cap, dtype=torch.float64)
    for _ in range(40):
        o, a, r, d, idx, w = bufs[1].sample_prioritized(8192)
        assert torch.all(o[:, 0].long() == idx)
        assert float(w.max()) <= 1.0 + 1e-6
        counts += torch.bincount(idx.cpu(), minlength=cap).double()
    p = pr.double() ** 0.6
    p /= p.sum()
    # chi-square over 50 equal-probability bins of the sorted leaves
    order = torch.argsort(p)
    bins = torch.tensor_split(order, 50)
    obs = torch.stack([counts[b].sum() for b in bins])
    exp = torch.stack([p[b].sum() for b in bins]) * counts.sum()
    chi2 = float(((obs - exp) ** 2 / exp).sum())
    assert chi2 < 49 + 6 * (2 * 49) ** 0.5
