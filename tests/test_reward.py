"""RewardEngine: the reference's RewardEngineTest cases
(turbol_vllm/tests/test_profiler_reward.cpp:118-233) and the token kernels."""
import pytest
import torch

import turbol_b200 as turbol
from turbol_b200.ops import reference as ref


def engine(**kw):
    c = turbol.RewardConfig()
    for k, v in kw.items():
        setattr(c, k, v)
    e = turbol.RewardEngine(c)
    assert e.initialize().ok()
    return e


def test_rule_scores_format_and_length():
    e = engine(normalize=False, format_bonus=0.5, length_penalty=-0.01, target_length=4)
    r = e.score_batch(["abcd.", "abcd", "ab"])
    rule = r.rule_scores.torch()
    assert torch.allclose(rule, torch.tensor([0.5 - 0.01, 0.0, -0.04]))
    assert torch.allclose(r.total.torch(), rule)
    assert torch.all(r.model_scores.torch() == 0) and torch.all(r.kl_penalties.torch() == 0)


def test_clip_and_normalize():
    e = engine(normalize=False, reward_clip=0.1, length_penalty=-1.0, target_length=0)
    r = e.score_batch(["aaaa"])
    assert float(r.total.torch()[0]) == pytest.approx(-0.1)
    e2 = engine(normalize=True)
    r2 = e2.score_batch(["a.", "bbbbbbbbb", "cc."])
    assert abs(float(r2.total.torch().mean())) < 1e-6


def test_adaptive_kl_direction():
    e = engine(adaptive_kl=True, kl_coef=0.1, kl_target=0.1, kl_adapt_rate=0.5)
    e.update_adaptive_kl(0.5)
    assert e.current_kl_coef() > 0.1
    e.update_adaptive_kl(-10.0)
    assert e.current_kl_coef() == 0.0
    f = engine(adaptive_kl=False, kl_coef=0.1)
    f.update_adaptive_kl(5.0)
    assert f.current_kl_coef() == pytest.approx(0.1)


def test_kl_penalty_and_token_scores_cpu():
    e = engine(kl_coef=0.5, normalize=False)
    lp = torch.tensor([[0.0, -1.0, -2.0], [-1.0, -1.0, 0.0]])
    rf = torch.tensor([[-1.0, -1.0, 0.0], [0.0, 0.0, 0.0]])
    m = torch.tensor([[1.0, 1.0, 0.0], [1.0, 1.0, 1.0]])
    kl = e.kl_penalty(lp, rf, m)
    assert torch.allclose(kl, torch.tensor([0.5 * 0.5, 0.5 * (-2 / 3)]))
    ids = torch.tensor([[1, 2, 46], [3, 4, 5]], dtype=torch.int32)
    res = e.score_tokens(turbol.from_torch(ids), turbol.from_torch(m), turbol.from_torch(rf), turbol.from_torch(lp))
    assert res.kl_penalties.torch().shape == (2,)


def test_welford_stats():
    e = engine()
    x = torch.randn(1000)
    e.update_stats(turbol.from_torch(x))
    assert e.running_count() == 1000
    assert abs(e.running_mean() - float(x.mean())) < 1e-6
    assert abs(e.running_var() - float(x.var(unbiased=False))) < 1e-5


def test_hash_reward_cpu_oracle():
    e = engine()
    ids = torch.randint(0, 151936, (16, 40), dtype=torch.int32)
    lens = torch.randint(1, 41, (16,), dtype=torch.int32)
    got = e.hash_reward(ids, lens)
    assert torch.allclose(got, ref.fnv1a_reward(ids, lens))
    assert torch.all((got >= 0) & (got < 1))


@pytest.mark.gpu
def test_reward_kernels_match_cpu(dev):
    e = engine(kl_coef=0.3, normalize=False, k3_kl=True)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 151936, (512, 512), dtype=torch.int32, generator=g)
    lens = torch.randint(1, 513, (512,), dtype=torch.int32, generator=g)
    assert torch.equal(e.hash_reward(ids.to(dev), lens.to(dev)).cpu(), e.hash_reward(ids, lens))
    lp = -torch.rand(64, 100, generator=g)
    rf = -torch.rand(64, 100, generator=g)
    m = (torch.rand(64, 100, generator=g) < 0.8).float()
    assert torch.allclose(e.kl_penalty(lp.to(dev), rf.to(dev), m.to(dev)).cpu(), e.kl_penalty(lp, rf, m), atol=1e-5)
    ids2 = torch.randint(0, 259, (64, 100), dtype=torch.int32, generator=g)
    rc = e.score_tokens(turbol.from_torch(ids2), turbol.from_torch(m))
    rg = e.score_tokens(turbol.from_torch(ids2.to(dev)), turbol.from_torch(m.to(dev)))
    assert torch.allclose(rc.total.torch(), rg.total.torch().cpu(), atol=1e-5)
    n = engine(normalize=True, whiten=True)
    r = n.score_tokens(turbol.from_torch(ids2.to(dev)), turbol.from_torch(m.to(dev))).total.torch()
    assert abs(float(r.mean())) < 1e-4
