"""Tensor-core actor-critic (hand-written forward/backward on the tcgen05 GEMM)
vs the fp32 autograd ActorCritic with identical weights."""
import pytest
import torch

from turbol_b200._native import ops
from turbol_b200.models.fused_mlp import FusedActorCritic
from turbol_b200.models.mlp import ActorCritic

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,B", [(256, 1000), (64, 4096), (128, 300)])
def test_fused_mlp_matches_autograd(H, B, dev):
    net = FusedActorCritic(4, 2, (H, H), device=dev, seed=3)
    ref = ActorCritic(4, 2, (H, H), discrete=True, device="cpu", seed=3)
    a, c = net.to_actor_critic_params()
    for p, q in zip(a + c, ref.actor_params + ref.critic_params):
        assert torch.allclose(p.cpu(), q, atol=1e-6)
    g = torch.Generator().manual_seed(B)
    obs = torch.randn(B, 4, generator=g) * 0.5
    x = torch.zeros(B, 8, device=dev, dtype=torch.bfloat16)
    ops().pad_obs_bf16(obs.to(dev).contiguous(), x)
    ws = net.workspace(B)
    logits, value = net.forward(x, ws)
    # reference on the bf16-rounded inputs, fp32 math
    xo = x[:, :4].float().cpu().requires_grad_()
    rl, rv = ref(xo)
    assert torch.allclose(logits[:, :2].cpu(), rl, atol=3e-2, rtol=3e-2)
    assert torch.allclose(value[:, 0].cpu(), rv, atol=3e-2, rtol=3e-2)
    # backward with the same upstream gradients
    dl = (torch.randn(B, 2, generator=g) / B).to(torch.bfloat16)
    dv = (torch.randn(B, generator=g) / B).to(torch.bfloat16)
    ws["dlog"].zero_()
    ws["dval"].zero_()
    ws["dlog"][:, :2].copy_(dl.to(dev))
    ws["dval"][:, 0].copy_(dv.to(dev))
    net.backward(x, ws)
    torch.autograd.backward([rl, rv], [dl.float(), dv.float()])
    ga = [net.g["w1"][:H, :4], net.g["b1"][:H], net.g["w2a"], net.g["b2a"], net.g["w3a"][:2], net.g["b3a"][:2]]
    gc = [net.g["w1"][H:, :4], net.g["b1"][H:], net.g["w2c"], net.g["b2c"], net.g["w3c"][:1], net.g["b3c"][:1]]
    for got, p in zip(ga + gc, ref.actor_params + ref.critic_params):
        exp = p.grad
        scale = float(exp.abs().max()) + 1e-8
        err = float((got.cpu() - exp).abs().max()) / scale
        assert err < 5e-2, (p.shape, err)
    # padding stays untouched by the gradients
    assert float(net.g["w1"][:, 4:].abs().max()) == 0.0
    assert float(net.g["w3a"][2:].abs().max()) == 0.0


def test_dense_k8_kernels(dev):
    from turbol_b200._native import ops
    o = ops()
    g = torch.Generator().manual_seed(4)
    M, N = 5000, 512
    x = torch.zeros(M, 8)
    x[:, :4] = torch.randn(M, 4, generator=g)
    x = x.to(dev, torch.bfloat16)
    W = (torch.randn(N, 8, generator=g) * 0.5).to(dev, torch.bfloat16)
    b = torch.randn(N, generator=g).to(dev)
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    o.dense_k8_fwd(x, W, b, y, True)
    ref = torch.tanh(x.float() @ W.float().t() + b)
    assert (y.float() - ref).abs().max().item() < 1e-2
    dz = torch.randn(M, N, generator=g).to(dev, torch.bfloat16)
    dW = torch.full((N, 8), 7.0, device=dev)
    o.dense_k8_wgrad(dz, x, dW)
    exp = dz.float().t() @ x.float()
    assert torch.allclose(dW, exp, atol=1e-2, rtol=1e-3)
    o.dense_k8_wgrad(dz, x, dW, True)
    assert torch.allclose(dW, 2 * exp, atol=2e-2, rtol=1e-3)


@pytest.mark.parametrize("N,xblock", [(512, 256), (512, 512), (128, 64), (256, 256)])
def test_skinny8_wgrad(N, xblock, dev):
    """out = A^T X per column block against fp32 torch, both output layouts."""
    o = ops()
    g = torch.Generator().manual_seed(N + xblock)
    M = 33333
    nb = N // xblock
    A = torch.randn(M, N, generator=g).to(dev, torch.bfloat16)
    X = torch.randn(M, 8 * nb, generator=g).to(dev, torch.bfloat16)
    exp = torch.zeros(8 * nb, N)  # [k + 8b, j]
    for b in range(nb):
        cols = slice(b * xblock, (b + 1) * xblock)
        exp[8 * b:8 * b + 8, cols] = X.float().cpu()[:, 8 * b:8 * b + 8].t() @ A.float().cpu()[:, cols]
    sc = torch.empty(o.skinny8_scratch_numel(N), device=dev)
    out = torch.zeros(8 * nb, N, device=dev)                # rows k + 8b, columns j (the w3 layout)
    out[:, :] = torch.where(exp != 0, 3.0, 0.0).to(dev)     # stale values where the kernel stores
    o.skinny8_wgrad(A, X, out, xblock, 1, N, 8 * N, False, sc)
    assert torch.allclose(out.cpu(), exp, atol=0.5, rtol=1e-3), (out.cpu() - exp).abs().max()
    if nb == 1:
        out2 = torch.zeros(N, 8, device=dev)                # [j, k] (the w1 layout)
        o.skinny8_wgrad(A, X, out2, xblock, 8, 1, 0, False, sc)
        o.skinny8_wgrad(A, X, out2, xblock, 8, 1, 0, True, sc)  # accumulate
        assert torch.allclose(out2.cpu(), 2 * exp.t(), atol=1.0, rtol=1e-3)


@pytest.mark.parametrize("N,xblock", [(512, 256), (128, 64), (256, 256)])
def test_mlp_head_dz(N, xblock, dev):
    """dZ = (dOut_head W_head) * (1 - H^2) and db = column sums, against fp32 torch."""
    o = ops()
    g = torch.Generator().manual_seed(N)
    M, nb = 20001, N // xblock
    dout = (torch.randn(M, 8 * nb, generator=g) * 0.1).to(dev, torch.bfloat16)
    h = torch.tanh(torch.randn(M, N, generator=g)).to(dev, torch.bfloat16)
    W = (torch.randn(8 * nb, N, generator=g) * 0.2).to(dev, torch.bfloat16)
    dz = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    db = torch.full((N,), 5.0, device=dev)
    sc = torch.empty(o.skinny8_scratch_numel(N), device=dev)
    o.mlp_head_dz(dout, h, W, xblock, dz, db, False, sc)
    pre = torch.zeros(M, N, device=dev)
    for b in range(nb):
        cols = slice(b * xblock, (b + 1) * xblock)
        pre[:, cols] = dout.float()[:, 8 * b:8 * b + 8] @ W.float()[8 * b:8 * b + 8, cols]
    exp = pre * (1 - h.float() ** 2)
    assert torch.allclose(dz.float(), exp, atol=1e-2, rtol=1e-2), (dz.float() - exp).abs().max()
    assert torch.allclose(db, exp.sum(0), atol=0.05, rtol=1e-3), (db - exp.sum(0)).abs().max()


@pytest.mark.parametrize("H", [256, 128, 64])
def test_mlp_head_fwd(H, dev):
    """out[:, 8b + k] = bias + H2_head . W3[8b + k] per head, against fp32 torch (row count not a multiple of 32)."""
    o = ops()
    g = torch.Generator().manual_seed(H)
    M = 10007
    h = torch.tanh(torch.randn(M, 2 * H, generator=g)).to(dev, torch.bfloat16)
    W = (torch.randn(16, 2 * H, generator=g) * 0.1).to(dev, torch.bfloat16)
    b = torch.randn(16, generator=g).to(dev)
    out = torch.full((M, 16), 7.0, device=dev)
    o.mlp_head_fwd(h, W, b, H, out)
    exp = torch.cat([h.float()[:, :H] @ W.float()[:8, :H].t(), h.float()[:, H:] @ W.float()[8:, H:].t()], 1) + b
    assert torch.allclose(out, exp, atol=2e-3, rtol=1e-3), (out - exp).abs().max()


@pytest.mark.parametrize("H,B", [(256, 3000), (128, 4099)])
def test_fused_ppo_head_matches_autograd(H, B, dev):
    """Hidden layers + the one-pass output layer / clipped PPO loss / output-layer
    backward (ppo_head.cu) + the hidden backward, against fp32 autograd of the
    same actor-critic and the reference loss expression: every parameter's
    gradient and the loss statistics."""
    from turbol_b200.ops import reference as refops

    net = FusedActorCritic(4, 2, (H, H), device=dev, seed=5)
    ref = ActorCritic(4, 2, (H, H), discrete=True, device="cpu", seed=5)
    g = torch.Generator().manual_seed(B + H)
    obs = torch.randn(B, 4, generator=g) * 0.5
    x = torch.zeros(B, 8, device=dev, dtype=torch.bfloat16)
    ops().pad_obs_bf16(obs.to(dev).contiguous(), x)
    xo = x[:, :4].float().cpu().requires_grad_()
    rl, rv = ref(xo)
    act = torch.randint(0, 2, (B,), generator=g, dtype=torch.int32)
    # behaviour log-probs near the current ones: some ratios fall outside the clip range
    old = (torch.log_softmax(rl.detach(), -1).gather(1, act.long()[:, None])[:, 0]
           + 0.3 * torch.randn(B, generator=g))
    adv = torch.randn(B, generator=g)
    ret = torch.randn(B, generator=g)
    loss, st_ref = refops.ppo_categorical_loss(rl, rv, act, old, adv, ret, 0.2, 0.5, 0.01)
    loss.backward()
    ws = net.workspace(B)
    stats = torch.zeros(8, device=dev)
    net.grad.fill_(0.0)
    net.forward_hidden(x, ws)
    net.loss_backward(x, ws, act.to(dev), old.to(dev), adv.to(dev), ret.to(dev), stats, 0.2, 0.5, 0.01)
    torch.cuda.synchronize()
    ga = [net.g["w1"][:H, :4], net.g["b1"][:H], net.g["w2a"], net.g["b2a"], net.g["w3a"][:2], net.g["b3a"][:2]]
    gc = [net.g["w1"][H:, :4], net.g["b1"][H:], net.g["w2c"], net.g["b2c"], net.g["w3c"][:1], net.g["b3c"][:1]]
    for got, p in zip(ga + gc, ref.actor_params + ref.critic_params):
        exp = p.grad
        scale = float(exp.abs().max()) + 1e-8
        err = float((got.cpu() - exp).abs().max()) / scale
        assert err < 5e-2, (p.shape, err)
    # gradients of the padding and of the off-diagonal blocks stay zero
    assert float(net.g["w3a"][2:].abs().max()) == 0.0 and float(net.g["w3c"][1:].abs().max()) == 0.0
    assert float(net.g["w3"][:8, H:].abs().max()) == 0.0 and float(net.g["w3"][8:, :H].abs().max()) == 0.0
    # statistics: [pg, v, entropy, kl, clipfrac] sums and the row count
    st = stats.cpu()
    assert st[5].item() == B
    for k in range(5):
        assert abs(st[k].item() - st_ref[k].item()) <= 2e-2 * max(1.0, abs(st_ref[k].item())), (k, st, st_ref)
