"""PPO: fused loss kernel and Adam kernel vs autograd/fp32 oracles; the
on-device permutation; end-to-end learning on CPU and GPU."""
import pytest
import torch

import turbol_b200 as turbol
from turbol_b200._native import ops
from turbol_b200.ops import reference as ref
from turbol_b200.ops.rl import FusedAdam, ppo_categorical_loss
from turbol_b200.rl.ppo import PPOConfig, PPOTrainer


def test_ppo_cpu_learns_cartpole():
    cfg = PPOConfig(num_envs=64, rollout_steps=32, minibatch_size=256, hidden=(64, 64), seed=1)
    tr = PPOTrainer(cfg, device="cpu")
    first = None
    for i in range(25):
        tr.train_iteration()
        if i == 2:
            first = tr.metrics()["mean_return"]
    tr.metrics()
    for _ in range(3):
        tr.train_iteration()
    last = tr.metrics()["mean_return"]
    assert last > 2 * first and last > 60, (first, last)


@pytest.mark.parametrize("hidden,ent", [((64, 64), 0.0), ((32,), 0.01)])
def test_cpu_ppo_host_minibatch_matches_autograd(hidden, ent):
    """The CPU trainer's minibatch step in the core (no autograd) gives the
    same update and loss statistics as the autograd path."""
    cfg = PPOConfig(num_envs=64, rollout_steps=8, hidden=hidden, epochs=2, minibatch_size=64, seed=2, ent_coef=ent)
    a = PPOTrainer(cfg, device="cpu")
    b = PPOTrainer(cfg, device="cpu")
    b.host_update = False
    for t in (a, b):
        t._rollout_cpu()
    assert torch.equal(a.obs_buf, b.obs_buf) and torch.equal(a.adv, b.adv)
    c = PPOTrainer(cfg, device="cpu")  # host minibatch steps, driven from Python one at a time
    c.grad_sync = lambda g: 1.0
    c._rollout_cpu()
    for t in (a, b, c):
        t._update_cpu()
    for t in (b, c):
        assert torch.allclose(a.policy.fp.flat, t.policy.fp.flat, atol=2e-6, rtol=1e-5), \
            (a.policy.fp.flat - t.policy.fp.flat).abs().max()
        assert torch.allclose(a.loss_stats, t.loss_stats, atol=1e-3, rtol=1e-4), (a.loss_stats, t.loss_stats)
    assert a.opt._host_step == b.opt._host_step == c.opt._host_step == cfg.epochs * cfg.n_minibatches


@pytest.mark.parametrize("hidden,B,scale,threads", [((64, 64), 64, 1.0, 1), ((20, 37), 13, 0.3, 1),
                                                    ((48,), 7, 4.0, 1), ((), 5, 1.0, 1), ((96, 80), 601, 1.0, 4)])
def test_host_minibatch_gradient_matches_fp64_autograd(hidden, B, scale, threads):
    """The core's minibatch step (register-tiled products, vector tanh)
    against float64 autograd of the same actor / critic MLPs and PPO loss:
    widths that are not multiples of the vector width, row counts that are not
    multiples of 4, saturated (scale 4) and near-linear (scale 0.3) hidden
    layers, and a minibatch large enough to be split over 4 threads."""
    from turbol_b200._native import core
    g = torch.Generator().manual_seed(3)
    O, A, N = 4, 3, max(97, B + 11)
    clip, vf, ent = 0.2, 0.5, 0.01
    dims_a, dims_c = [O, *hidden, A], [O, *hidden, 1]
    parts = []
    for dims in (dims_a, dims_c):
        for i, o in zip(dims[:-1], dims[1:]):
            parts += [torch.randn(o * i, generator=g) * scale / i ** 0.5, torch.randn(o, generator=g) * 0.1]
    flat = torch.cat(parts)
    obs = torch.randn(N, O, generator=g) * 2
    act = torch.randint(0, A, (N,), generator=g, dtype=torch.int32)
    old_logp = torch.randn(N, generator=g) * 0.3 - 1.1
    adv, ret = torch.randn(N, generator=g), torch.randn(N, generator=g)
    idx = torch.randperm(N, generator=g)[:B]
    grad, stats = torch.zeros_like(flat), torch.zeros(6)
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        core().ppo_minibatch_host(flat, grad, dims_a, dims_c, obs, act, old_logp, adv, ret, idx, clip, vf, ent, stats)
    finally:
        torch.set_num_threads(prev)

    p64 = flat.double().requires_grad_()
    x = obs[idx].double()

    def mlp(dims, off):
        h = x
        for li, (i, o) in enumerate(zip(dims[:-1], dims[1:])):
            W = p64[off:off + o * i].view(o, i)
            b = p64[off + o * i:off + o * i + o]
            off += o * i + o
            h = h @ W.t() + b
            if li + 2 < len(dims):
                h = torch.tanh(h)
        return h, off

    logits, off = mlp(dims_a, 0)
    value = mlp(dims_c, off)[0].squeeze(1)
    lp_all = torch.log_softmax(logits, -1)
    lp = lp_all.gather(1, act[idx].long().view(-1, 1)).squeeze(1)
    ratio = torch.exp(lp - old_logp[idx].double())
    a_, r_ = adv[idx].double(), ret[idx].double()
    pg = -torch.min(ratio * a_, ratio.clamp(1 - clip, 1 + clip) * a_)
    entropy = -(lp_all.exp() * lp_all).sum(-1)
    loss = pg.mean() + vf * (0.5 * (value - r_) ** 2).mean() - ent * entropy.mean()
    loss.backward()
    assert torch.allclose(grad.double(), p64.grad, rtol=1e-4, atol=1e-6), (grad.double() - p64.grad).abs().max()
    assert abs(stats[0].item() - pg.sum().item()) < 1e-4 * max(1.0, abs(pg.sum().item()))
    assert abs(stats[2].item() - entropy.sum().item()) < 1e-4 * entropy.sum().item() and stats[5].item() == B


def test_cpu_host_rollout_matches_policy_and_environment():
    """The one-call CPU rollout (ppo_cartpole_rollout_host): the recorded
    observations replay bit-exactly through a second environment stepped with
    the recorded actions; log-probabilities and values equal the torch
    policy's; the actions follow the policy's probabilities; the same seed and
    iteration give the same rollout."""
    cfg = PPOConfig(num_envs=256, rollout_steps=16, hidden=(32, 24), seed=4)
    tr = PPOTrainer(cfg, device="cpu")
    with torch.no_grad():  # a policy that is not near-uniform, so the sampling test has power
        tr.policy.actor_params[-2].mul_(60.0)
    s0 = tr.state.clone()
    tr._rollout_cpu()
    T, N = cfg.rollout_steps, cfg.num_envs
    assert torch.equal(tr.obs_buf[0], s0)
    env = turbol.GPUEnvironment(N, 4, 2, "cpu", "cartpole", seed=tr.env.seed())
    assert torch.equal(env.state(), s0)
    obs, rew, done = torch.empty(N, 4), torch.empty(N), torch.empty(N, dtype=torch.uint8)
    for t in range(T):
        env.step_into(tr.act_buf[t], obs, rew, done)
        assert torch.equal(obs, tr.obs_buf[t + 1] if t + 1 < T else tr.state), t
        assert torch.equal(rew, tr.rew_buf[t]) and torch.equal(done, tr.done_buf[t]), t
    with torch.no_grad():
        logits, v = tr.policy(tr.obs_buf.view(T * N, 4))
        lp_all = torch.log_softmax(logits, -1)
        lp = lp_all.gather(1, tr.act_buf.view(-1, 1).long()).squeeze(1)
        assert torch.allclose(lp, tr.logp_buf.view(-1), atol=2e-5, rtol=1e-5)
        assert torch.allclose(v, tr.val_buf[:T].reshape(-1), atol=2e-5, rtol=1e-5)
        assert torch.allclose(tr.policy.critic(tr.state), tr.val_buf[T], atol=2e-5, rtol=1e-5)
    p1 = lp_all[:, 1].exp().double()
    n1 = (tr.act_buf == 1).sum().item()
    sd = (p1 * (1 - p1)).sum().sqrt().item()
    assert 0.02 < p1.mean().item() < 0.98 and abs(n1 - p1.sum().item()) < 5 * sd, (n1, p1.sum().item(), sd)
    again = PPOTrainer(cfg, device="cpu")
    with torch.no_grad():
        again.policy.actor_params[-2].mul_(60.0)
    again._rollout_cpu()
    for name in ("obs_buf", "act_buf", "logp_buf", "val_buf", "rew_buf", "done_buf"):
        assert torch.equal(getattr(tr, name), getattr(again, name)), name


def test_cpu_host_rollout_is_the_same_on_any_thread_count():
    """A rollout large enough to be split by rows over threads (1,024 envs,
    MLP 128-128) gives bit-identical buffers with 1 and with 4 intra-op
    threads: each row's forward and draw depend on that row only.  (Both
    trainers are built under the same thread count: the orthogonal
    initialization itself rounds differently on different counts.)"""
    cfg = PPOConfig(num_envs=1024, rollout_steps=4, hidden=(128, 128), seed=6)
    out = [PPOTrainer(cfg, device="cpu") for _ in range(2)]
    assert torch.equal(out[0].policy.fp.flat, out[1].policy.fp.flat)
    prev = torch.get_num_threads()
    try:
        for tr, threads in zip(out, (1, 4)):
            torch.set_num_threads(threads)
            tr._rollout_cpu()
    finally:
        torch.set_num_threads(prev)
    for name in ("obs_buf", "act_buf", "logp_buf", "val_buf", "rew_buf", "done_buf"):
        assert torch.equal(getattr(out[0], name), getattr(out[1], name)), name


def test_policy_engine_reference_api():
    pe = turbol.PolicyEngine(obs_dim=4, act_dim=2, device="cpu")
    assert pe.initialize().ok()
    obs = turbol.Tensor([8, 4], "float32", "cpu")
    a, lp = turbol.Tensor(), turbol.Tensor()
    assert pe.forward(obs, a, lp).ok()
    assert a.shape().to_list() == [8, 2] and lp.shape().to_list() == [8]
    assert float(a.torch().abs().max()) <= 1.0
    v = turbol.Tensor()
    assert pe.get_value(obs, v).ok() and v.shape().to_list() == [8]
    act, logp = pe.forward(obs)  # README form
    batch = torch.randn(8, 4 + 2 + 2)
    before = pe.net.fp.flat.clone()
    assert pe.update(turbol.from_torch(batch)).ok()
    assert not torch.equal(before, pe.net.fp.flat)


@pytest.mark.parametrize("has_old", [False, True])
def test_policy_engine_host_linear_gaussian_matches_autograd(has_old):
    """On the CPU the linear Gaussian model acts and computes its gradient in
    the core's host loops; the update equals the autograd path's, the log-prob
    is the Gaussian density of the sample, and the noise is standard normal."""
    O, A, N = 16, 4, 300
    host = turbol.PolicyEngine(obs_dim=O, act_dim=A, device="cpu", seed=3)
    eager = turbol.PolicyEngine(obs_dim=O, act_dim=A, device="cpu", seed=3)
    host.initialize()
    eager.initialize()
    eager._host_fused = lambda: False
    assert host._host_fused()
    g = torch.Generator().manual_seed(5)
    obs = torch.randn(N, O, generator=g)
    act = (torch.rand(N, A, generator=g) * 2 - 1) * 0.9
    adv, ret = torch.randn(N, 1, generator=g), torch.randn(N, 1, generator=g)
    cols = [obs, act, adv, ret]
    if has_old:
        cols.append(torch.randn(N, 1, generator=g) * 0.3 - 4.0)
    batch = torch.cat(cols, 1)
    for _ in range(3):
        assert host.update(batch).ok() and eager.update(batch).ok()
    assert torch.allclose(host.net.fp.flat, eager.net.fp.flat, atol=2e-5, rtol=1e-4), \
        (host.net.fp.flat - eager.net.fp.flat).abs().max()
    x = torch.randn(4096, O)
    a, lp = host.act(x)
    assert a.shape == (4096, A) and lp.shape == (4096,) and float(a.abs().max()) <= 1.0
    with torch.no_grad():
        mean = host.net.actor(x)
        assert torch.allclose(lp, host.net.gaussian_logprob(mean, a), atol=1e-4, rtol=1e-4)
    assert not torch.equal(a, host.act(x)[0])
    narrow = turbol.PolicyEngine(obs_dim=O, act_dim=A, device="cpu", seed=4, std=0.05)
    narrow.initialize()
    z = narrow.act(torch.zeros(1 << 15, O))[0] / 0.05
    assert abs(float(z.mean())) < 0.03 and abs(float(z.std()) - 1.0) < 0.03
    assert abs(float((z.abs() < 1).float().mean()) - 0.6827) < 0.015


def test_host_adam_matches_the_oracle():
    from turbol_b200.ops import reference as ref

    n = 1001
    g0 = torch.Generator().manual_seed(1)
    p = torch.randn(n, generator=g0)
    opt = FusedAdam(p.clone(), torch.zeros(n), lr=1e-3, weight_decay=0.01)
    pr, mr, vr = p.clone().double(), torch.zeros(n, dtype=torch.float64), torch.zeros(n, dtype=torch.float64)
    for step in range(1, 5):
        grad = torch.randn(n, generator=g0)
        opt.g.copy_(grad)
        opt.step(grad_scale=0.5)
        ref.adam_step(pr, grad.double(), mr, vr, step, 1e-3, wd=0.01, grad_scale=0.5)
        assert torch.allclose(opt.p.double(), pr, atol=1e-6), step


def test_policy_engine_discrete_ppo_update():
    pe = turbol.PolicyEngine(obs_dim=4, act_dim=2, device="cpu", hidden=(32,), discrete=True)
    pe.initialize()
    obs = torch.randn(16, 4)
    act, logp = pe.forward(obs)
    batch = torch.cat([obs, act[:, None].float(), torch.randn(16, 1), torch.randn(16, 1), logp[:, None]], 1)
    assert pe.update(batch).ok()


@pytest.mark.gpu
@pytest.mark.parametrize("A", [2, 3, 8])
def test_ppo_loss_kernel_grads(A, dev):
    B = 5000
    g = torch.Generator().manual_seed(A)
    logits = torch.randn(B, A, generator=g)
    value = torch.randn(B, generator=g)
    act = torch.randint(0, A, (B,), generator=g, dtype=torch.int32)
    old = torch.log_softmax(logits + 0.3 * torch.randn(B, A, generator=g), -1).gather(1, act.long()[:, None]).squeeze(1)
    adv = torch.randn(B, generator=g)
    ret = torch.randn(B, generator=g)
    lr_, vr = logits.clone().double().requires_grad_(), value.clone().double().requires_grad_()
    loss, st = ref.ppo_categorical_loss(lr_, vr, act, old.double(), adv.double(), ret.double(), 0.2, 0.5, 0.01)
    loss.backward()
    stats = torch.zeros(8, device=dev)
    lg = logits.to(dev).requires_grad_()
    vg = value.to(dev).requires_grad_()
    out = ppo_categorical_loss(lg, vg, act.to(dev), old.to(dev), adv.to(dev), ret.to(dev), 0.2, 0.5, 0.01,
                               stats=stats)
    out.backward()
    assert torch.allclose(lg.grad.cpu().double(), lr_.grad, atol=1e-6, rtol=1e-4)
    assert torch.allclose(vg.grad.cpu().double(), vr.grad, atol=1e-7, rtol=1e-4)
    s = stats.cpu().double()
    assert torch.allclose(s[:6], st.double(), rtol=1e-3, atol=1e-2)


@pytest.mark.gpu
def test_adam_kernel_matches_reference(dev):
    n = 100003
    g = torch.Generator().manual_seed(0)
    p = torch.randn(n, generator=g)
    opt = FusedAdam(p.clone().to(dev), torch.zeros(n, device=dev), lr=1e-3, weight_decay=0.01, bf16_shadow=True)
    pr, m, v = p.clone().double(), torch.zeros(n, dtype=torch.float64), torch.zeros(n, dtype=torch.float64)
    for step in range(1, 6):
        grad = torch.randn(n, generator=g)
        opt.g.copy_(grad.to(dev))
        opt.step(grad_scale=0.5)
        ref.adam_step(pr, grad.double(), m, v, step, 1e-3, 0.9, 0.999, 1e-8, 0.01, 0.5)
    assert torch.allclose(opt.p.cpu().double(), pr, atol=1e-6)
    assert torch.allclose(opt.shadow.float().cpu(), opt.p.cpu(), rtol=1e-2, atol=1e-3)
    assert int(opt.step_t.item()) == 5


@pytest.mark.gpu
def test_gather_permutation_covers_batch(dev):
    T, N, MB = 8, 512, 1024
    total = T * N
    obs = torch.arange(total * 4, dtype=torch.float32, device=dev).view(T, N, 4)
    act = torch.arange(total, dtype=torch.int32, device=dev).view(T, N)
    f = torch.arange(total, dtype=torch.float32, device=dev).view(T, N)
    outs = [torch.empty(MB, 4, device=dev), torch.empty(MB, dtype=torch.int32, device=dev)] + \
        [torch.empty(MB, device=dev) for _ in range(3)]
    seen = []
    n_mb = total // MB
    for step in range(n_mb):
        ops().ppo_gather(obs, act, f, f, f, f, None, outs[0], outs[1], outs[2], outs[3], outs[4], None, n_mb, None,
                         None, step, 1234, False)
        seen.append(outs[1].cpu().clone())
        assert torch.equal(outs[0][:, 0].long().cpu(), outs[1].long().cpu() * 4)
        assert torch.equal(outs[2].cpu(), outs[1].float().cpu())
    allidx = torch.cat(seen)
    assert torch.equal(torch.sort(allidx).values, torch.arange(total, dtype=torch.int32))
    assert not torch.equal(allidx, torch.arange(total, dtype=torch.int32))  # actually shuffled


@pytest.mark.gpu
@pytest.mark.parametrize("graphs", [False, True])
def test_ppo_gpu_learns(graphs, dev):
    cfg = PPOConfig(num_envs=1024, rollout_steps=32, minibatch_size=2048, hidden=(64, 64), seed=1,
                    cuda_graphs=graphs)
    tr = PPOTrainer(cfg, device=dev)
    tr.train_iteration()
    first = tr.metrics()["mean_return"]
    for _ in range(30):
        tr.train_iteration()
    tr.metrics()
    for _ in range(3):
        tr.train_iteration()
    m = tr.metrics()
    tr.release_graphs()
    assert m["mean_return"] > 2 * first and m["mean_return"] > 80, (first, m)
    assert 0 <= m["clipfrac"] <= 1 and m["entropy"] > 0


@pytest.mark.gpu
@pytest.mark.parametrize("has_old", [False, True])
def test_policy_engine_fused_linear_gaussian_matches_autograd(has_old, dev):
    """The fused act / gradient kernels of the linear Gaussian model give the
    same update as the autograd path, and consistent samples."""
    O, A, N = 16, 4, 300
    fused = turbol.PolicyEngine(obs_dim=O, act_dim=A, device=dev, seed=3)
    eager = turbol.PolicyEngine(obs_dim=O, act_dim=A, device=dev, seed=3)
    fused.initialize()
    eager.initialize()
    eager._fused = lambda: False
    assert fused._fused()
    g = torch.Generator().manual_seed(5)
    obs = torch.randn(N, O, generator=g)
    act = (torch.rand(N, A, generator=g) * 2 - 1) * 0.9
    adv, ret = torch.randn(N, 1, generator=g), torch.randn(N, 1, generator=g)
    cols = [obs, act, adv, ret]
    if has_old:
        cols.append(torch.randn(N, 1, generator=g) * 0.3 - 4.0)
    batch = torch.cat(cols, 1).to(dev)
    for _ in range(3):
        assert fused.update(batch).ok() and eager.update(batch).ok()
    torch.cuda.synchronize()
    assert torch.allclose(fused.net.fp.flat, eager.net.fp.flat, atol=2e-5, rtol=1e-4), \
        (fused.net.fp.flat - eager.net.fp.flat).abs().max()
    x = torch.randn(4096, O, device=dev)
    a, lp = fused.act(x)
    assert a.shape == (4096, A) and lp.shape == (4096,)
    assert float(a.abs().max()) <= 1.0
    mean = fused.net.actor(x)
    assert torch.allclose(lp, fused.net.gaussian_logprob(mean, a), atol=1e-4, rtol=1e-4)
    a2, _ = fused.act(x)
    assert not torch.equal(a, a2)
    # the noise is standard normal (zero observations -> zero mean; a small std keeps every sample unclamped)
    narrow = turbol.PolicyEngine(obs_dim=O, act_dim=A, device=dev, seed=4, std=0.05)
    narrow.initialize()
    z = narrow.act(torch.zeros(1 << 16, O, device=dev))[0] / 0.05
    assert abs(float(z.mean())) < 0.02 and abs(float(z.std()) - 1.0) < 0.02
    assert abs(float((z.abs() < 1).float().mean()) - 0.6827) < 0.01
