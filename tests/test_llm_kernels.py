"""LLM kernels vs plain fp32 PyTorch references."""
import math

import pytest
import torch
import torch.nn.functional as F

from turbol_b200._native import ops
from turbol_b200.models.llm import LMConfig, rope_table
from turbol_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def bf(x):
    return x.to(torch.bfloat16)


def test_rmsnorm_fwd_bwd(dev):
    T, D = 300, 1536
    x = bf(torch.randn(T, D, device=dev))
    w = torch.rand(D, device=dev) + 0.5
    y = torch.empty_like(x)
    r = torch.empty(T, device=dev)
    ops().rmsnorm_fwd(x, w, y, r, 1e-6)
    xr = x.float().requires_grad_()
    wr = w.clone().requires_grad_()
    yr = ref.rmsnorm(xr, wr, 1e-6)
    assert torch.allclose(y.float(), yr, atol=3e-2, rtol=2e-2)
    dy = bf(torch.randn(T, D, device=dev))
    add = bf(torch.randn(T, D, device=dev))
    dx = torch.empty_like(x)
    dw = torch.zeros(D, device=dev)
    ops().rmsnorm_bwd(dy, x, w, r, dx, add, dw)
    yr.backward(dy.float())
    assert torch.allclose(dx.float(), xr.grad + add.float(), atol=5e-2, rtol=3e-2)
    assert torch.allclose(dw, wr.grad, atol=0.5, rtol=2e-2)
    # the two-pass weight gradient (workspace) accumulates the same sum
    ws = torch.empty(ops().rmsnorm_bwd_ws_numel(D), device=dev)
    dw2 = torch.full((D,), 1.0, device=dev)
    dx2 = torch.empty_like(x)
    ops().rmsnorm_bwd(dy, x, w, r, dx2, add, dw2, ws)
    assert torch.equal(dx2, dx)
    assert torch.allclose(dw2 - 1.0, dw, atol=1e-2, rtol=1e-4)


def test_rope_roundtrip(dev):
    cfg = LMConfig.tiny()
    tab = rope_table(cfg, dev)
    T, Hh = 50, 6
    qkv = bf(torch.randn(T, Hh * 128, device=dev))
    pos = torch.randint(0, 500, (T,), device=dev, dtype=torch.int32)
    orig = qkv.clone()
    ops().rope(qkv, pos, tab, Hh, 128)
    x = orig.float().view(T, Hh, 128)
    ang = pos.double()[:, None] * (1.0 / cfg.rope_theta ** (torch.arange(0, 128, 2, device=dev).double() / 128))[None]
    c, s = torch.cos(ang).float()[:, None], torch.sin(ang).float()[:, None]
    e = torch.cat([x[..., :64] * c - x[..., 64:] * s, x[..., 64:] * c + x[..., :64] * s], -1)
    assert torch.allclose(qkv.float().view(T, Hh, 128), e, atol=3e-2)
    ops().rope(qkv, pos, tab, Hh, 128, True)
    assert torch.allclose(qkv.float(), orig.float(), atol=5e-2)


def test_rope_kv_write_matches_separate_kernels(dev):
    """The fused RoPE + paged KV write equals rope followed by kv_write, bit for bit."""
    cfg = LMConfig.tiny()
    tab = rope_table(cfg, dev)
    T, Hq, Hk, D, bs = 37, 6, 2, 128, 16
    qkv = bf(torch.randn(T, (Hq + 2 * Hk) * D + 64, device=dev))[:, :(Hq + 2 * Hk) * D]  # strided rows
    # distinct (sequence, position) per token: each cache slot is written once
    seq = (torch.arange(T, device=dev) % 5).to(torch.int32)
    pos = ((torch.arange(T, device=dev) // 5) * 37 + seq * 3).to(torch.int32)
    nblk = 5 * 20 + 1
    table = torch.randperm(nblk - 1, device=dev).to(torch.int32)[:5 * 20].view(5, 20)
    kc1 = bf(torch.zeros(nblk, Hk, bs, D, device=dev))
    vc1, kc2, vc2 = kc1.clone(), kc1.clone(), kc1.clone()
    a, b = qkv.clone(), qkv.clone()
    ops().rope(a, pos, tab, Hq + Hk, D)
    ops().kv_write(a, Hq * D, (Hq + Hk) * D, seq, pos, table, kc1, vc1, Hk, D, bs)
    ops().rope_kv_write(b, pos, tab, Hq, Hk, D, seq, table, kc2, vc2, bs)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)


@pytest.mark.parametrize("impl,use_ws", [("tc", True), ("tc", False), ("mma", False)])
@pytest.mark.parametrize("B,T,Hq,Hk", [(2, 128, 4, 2), (1, 200, 12, 2), (2, 64, 8, 8), (1, 777, 12, 2),
                                       (2, 320, 32, 8)])
def test_flash_attention_fwd_bwd(B, T, Hq, Hk, impl, use_ws, dev):
    """Forward + backward vs fp32 autograd.  impl 'tc' runs the tcgen05
    kernels (with a workspace the dK/dV pass splits GQA groups over CTAs and
    sums in fp32); 'mma' the mma.sync ones."""
    D = 128
    ld = (Hq + 2 * Hk) * D
    qkv = bf(torch.randn(B * T, ld, device=dev) * 0.5)
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D:(Hq + Hk) * D], qkv[:, (Hq + Hk) * D:]
    o = torch.empty(B * T, Hq * D, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(B * Hq * T, device=dev)
    scale = 1 / math.sqrt(D)
    ops().flash_attn_fwd(q, k, v, o, lse, B, T, Hq, Hk, scale, impl=impl)
    qr = q.float().view(B, T, Hq, D).requires_grad_()
    kr = k.float().view(B, T, Hk, D).requires_grad_()
    vr = v.float().view(B, T, Hk, D).requires_grad_()
    out = ref.causal_attention(qr, kr, vr, scale)
    assert torch.allclose(o.float().view(B, T, Hq, D), out, atol=2e-2, rtol=2e-2), (o.float().view(B, T, Hq, D) - out).abs().max()
    do = bf(torch.randn(B * T, Hq * D, device=dev))
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(B * Hq * T, device=dev)
    ws = torch.empty(ops().flash_attn_bwd_ws_numel(B, T, Hk), device=dev) if use_ws else None
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    dqkv.fill_(float("nan"))
    ops().flash_attn_bwd(q, k, v, o, do, lse, delta, dqkv[:, : Hq * D], dqkv[:, Hq * D:(Hq + Hk) * D],
                         dqkv[:, (Hq + Hk) * D:], B, T, Hq, Hk, scale, impl=impl, ws=ws,
                         err=err if impl == "tc" else None)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    out.backward(do.float().view(B, T, Hq, D))
    for got, exp in ((dqkv[:, : Hq * D], qr.grad), (dqkv[:, Hq * D:(Hq + Hk) * D], kr.grad),
                     (dqkv[:, (Hq + Hk) * D:], vr.grad)):
        e = exp.reshape(B * T, -1)
        err = (got.float() - e).abs().max() / (e.abs().max() + 1e-6)
        assert err < 3e-2, err


@pytest.mark.parametrize("B,T,Hq,Hk,amp", [(1, 64, 4, 2, 1.0), (2, 200, 12, 2, 1.0), (3, 333, 8, 8, 1.0),
                                          (1, 768, 12, 2, 3.0), (2, 300, 32, 8, 6.0)])
def test_flash_attention_fwd_tcgen05(B, T, Hq, Hk, amp, dev):
    """tcgen05 forward vs an fp32 reference and vs the mma.sync kernel (same LSE).
    amp > 1 makes the scores large and uneven, so the lazily updated row max
    moves mid-sequence and the O accumulator in TMEM gets rescaled."""
    D = 128
    ld = (Hq + 2 * Hk) * D
    g = torch.Generator(device=dev).manual_seed(T + Hq)
    qkv = bf(torch.randn(B * T, ld, device=dev, generator=g) * 0.5)
    qkv[:, : Hq * D] *= amp
    # a ramp on the keys: later keys score higher, so the running max keeps growing
    ramp = torch.linspace(0, amp, T, device=dev).repeat(B)[:, None]
    qkv[:, Hq * D:(Hq + Hk) * D] = bf(qkv[:, Hq * D:(Hq + Hk) * D].float() + ramp)
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D:(Hq + Hk) * D], qkv[:, (Hq + Hk) * D:]
    scale = 1 / math.sqrt(D)
    o_tc = torch.full((B * T, Hq * D), float("nan"), device=dev, dtype=torch.bfloat16)
    lse_tc = torch.full((B * Hq * T,), float("nan"), device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops().flash_attn_fwd(q, k, v, o_tc, lse_tc, B, T, Hq, Hk, scale, impl="tc", err=err)
    o_mma = torch.empty_like(o_tc)
    lse_mma = torch.empty_like(lse_tc)
    ops().flash_attn_fwd(q, k, v, o_mma, lse_mma, B, T, Hq, Hk, scale, impl="mma")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    out = ref.causal_attention(q.float().view(B, T, Hq, D), k.float().view(B, T, Hk, D),
                               v.float().view(B, T, Hk, D), scale)
    got = o_tc.float().view(B, T, Hq, D)
    assert torch.isfinite(got).all()
    assert (got - out).abs().max() < 3e-2 * max(1.0, out.abs().max().item())
    assert (got - o_mma.float().view(B, T, Hq, D)).abs().max() < 3e-2 * max(1.0, out.abs().max().item())
    assert torch.isfinite(lse_tc).all()
    assert torch.allclose(lse_tc, lse_mma, atol=2e-2, rtol=1e-3)


@pytest.mark.parametrize("n_split", [1, 3])
@pytest.mark.parametrize("Hq,Hk,bs", [(12, 2, 16), (32, 8, 16), (8, 1, 16), (4, 4, 16), (12, 2, 8)])
def test_decode_attention_paged(dev, Hq, Hk, bs, n_split):
    # bs 16 with up to 8 query heads per kv head runs the tensor-core kernel; bs 8 the CUDA-core one
    B, D = 5, 128
    lens = [1, 17, 33, 100, 64]
    nblk = 80
    kc = bf(torch.randn(nblk, Hk, bs, D, device=dev))
    vc = bf(torch.randn(nblk, Hk, bs, D, device=dev))
    perm = torch.randperm(nblk)
    table = torch.zeros(B, 16, dtype=torch.int32)
    used = 0
    for b in range(B):
        nb = (lens[b] + bs - 1) // bs
        table[b, :nb] = perm[used:used + nb].to(torch.int32)
        used += nb
    table = table.to(dev)
    # slots past each context hold garbage in a real cache: make it non-finite here
    for b in range(B):
        L = lens[b]
        if L % bs:
            kc[table[b, L // bs], :, L % bs:] = float("nan")
            vc[table[b, L // bs], :, L % bs:] = float("inf")
    q = bf(torch.randn(B, Hq * D, device=dev))
    out = torch.empty_like(q)
    ctx = torch.tensor(lens, device=dev, dtype=torch.int32)
    if n_split > 1:
        if bs != 16:
            pytest.skip("the context split is a mode of the tensor-core kernel (16-token blocks)")
        # chunks of the 1-block contexts are empty: the merge must skip them
        part = torch.full((ops().decode_attention_part_numel(B, Hq, Hk, n_split),), float("nan"), device=dev)
        cnt = torch.zeros(B * Hk, device=dev, dtype=torch.int32)
        for _ in range(2):  # the counters are left zero for the next call
            ops().decode_attention(q, kc, vc, table, ctx, out, Hq, Hk, D, bs, 1 / math.sqrt(D), n_split, part, cnt)
        torch.cuda.synchronize()
        assert int(cnt.abs().sum()) == 0
    else:
        ops().decode_attention(q, kc, vc, table, ctx, out, Hq, Hk, D, bs, 1 / math.sqrt(D))
    for b in range(B):
        L = lens[b]
        assert torch.isfinite(out[b].float()).all(), b
        ks = torch.cat([kc[table[b, j]].float() for j in range((L + bs - 1) // bs)], 1)[:, :L]  # [Hk, L, D]
        vs = torch.cat([vc[table[b, j]].float() for j in range((L + bs - 1) // bs)], 1)[:, :L]
        qq = q[b].float().view(Hq, D)
        kk = ks.repeat_interleave(Hq // Hk, 0)
        vv = vs.repeat_interleave(Hq // Hk, 0)
        p = torch.softmax((qq[:, None, :] * kk).sum(-1) / math.sqrt(D), -1)
        e = (p[..., None] * vv).sum(1)
        assert torch.allclose(out[b].float().view(Hq, D), e, atol=3e-2), b


def test_sample_and_logprob(dev):
    B, V = 7, 50000
    logits = bf(torch.randn(B, V, device=dev) * 3)
    tok = torch.empty(B, device=dev, dtype=torch.int32)
    lp = torch.empty(B, device=dev)
    ops().sample(logits, 0.0, 1, None, 0, tok, lp)  # greedy
    assert torch.equal(tok.long(), logits.float().argmax(-1))
    lsm = torch.log_softmax(logits.float(), -1)
    assert torch.allclose(lp, lsm.gather(1, tok.long()[:, None])[:, 0], atol=1e-3)
    # temperature sampling: empirical frequencies follow softmax
    small = bf(torch.tensor([[0.0, 1.0, 2.0, -1.0]] * 4096, device=dev))
    t = torch.empty(4096, device=dev, dtype=torch.int32)
    ops().sample(small, 1.0, 7, None, 3, t, None)
    freq = torch.bincount(t.long(), minlength=4).float() / 4096
    assert torch.allclose(freq.cpu(), torch.softmax(small[0].float(), -1).cpu(), atol=0.03)
    # vectorized rows (V % 8 == 0), temperature 0.7, log-probs of the sampled tokens
    row = torch.randn(1, 96) * 2
    wide = bf(row.repeat(16384, 1).to(dev))
    t2, lp2 = torch.empty(16384, device=dev, dtype=torch.int32), torch.empty(16384, device=dev)
    ops().sample(wide, 0.7, 11, None, 5, t2, lp2)
    p = torch.softmax(wide[0].float() / 0.7, -1)
    freq = torch.bincount(t2.long(), minlength=96).float() / 16384
    assert (freq - p).abs().max().item() < 0.02
    assert torch.allclose(lp2, p.log()[t2.long()], atol=1e-3)
    # log-probs and the in-place gradient
    tgt = torch.randint(0, V, (B,), device=dev, dtype=torch.int32)
    lg = logits.clone()
    out = torch.empty(B, device=dev)
    ops().logprob(lg, tgt, out)
    assert torch.allclose(out, lsm.gather(1, tgt.long()[:, None])[:, 0], atol=2e-3)
    g = torch.randn(B, device=dev)
    ops().logprob(lg, tgt, None, g)
    exp = g[:, None] * (F.one_hot(tgt.long(), V).float() - lsm.exp())
    assert torch.allclose(lg.float(), exp, atol=2e-3, rtol=1e-2)  # gradient stored in bf16


def test_grpo_loss_grad(dev):
    B, T = 6, 40
    lp = (-torch.rand(B, T, device=dev) * 3).requires_grad_()
    old = lp.detach() + 0.1 * torch.randn(B, T, device=dev)
    refl = lp.detach() + 0.2 * torch.randn(B, T, device=dev)
    adv = torch.randn(B, device=dev)
    mask = (torch.rand(B, T, device=dev) < 0.8).float()
    clip, beta = 0.2, 0.04
    r = torch.exp(lp - old)
    pg = -torch.min(r * adv[:, None], r.clamp(1 - clip, 1 + clip) * adv[:, None])
    d = refl - lp
    kl = torch.exp(d) - d - 1
    loss = (((pg + beta * kl) * mask).sum(1) / mask.sum(1)).sum() / B
    loss.backward()
    dlp = torch.empty(B, T, device=dev)
    stats = torch.zeros(4, device=dev)
    ops().grpo_loss(lp.detach().contiguous(), old, refl, adv, mask, dlp, stats, clip, beta, 1.0 / B)
    assert torch.allclose(dlp, lp.grad, atol=1e-6)
    assert abs(float(stats[0] + beta * stats[1]) - float(loss)) < 1e-4


def test_swiglu_and_embedding(dev):
    T, F_ = 33, 64
    gu = bf(torch.randn(T, 2 * F_, device=dev))
    act = torch.empty(T, F_, device=dev, dtype=torch.bfloat16)
    ops().swiglu_fwd(gu, act)
    g, u = gu.float()[:, 0::2].requires_grad_(), gu.float()[:, 1::2].requires_grad_()
    e = F.silu(g) * u
    assert torch.allclose(act.float(), e, atol=2e-2)
    dh = bf(torch.randn(T, F_, device=dev))
    dgu = torch.empty_like(gu)
    ops().swiglu_bwd(gu, dh, dgu)
    e.backward(dh.float())
    assert torch.allclose(dgu.float()[:, 0::2], g.grad, atol=3e-2)
    assert torch.allclose(dgu.float()[:, 1::2], u.grad, atol=3e-2)
    V, D = 100, 256
    W = bf(torch.randn(V, D, device=dev))
    ids = torch.randint(0, V, (77,), device=dev, dtype=torch.int32)
    out = torch.empty(77, D, device=dev, dtype=torch.bfloat16)
    ops().embed_fwd(ids, W, out)
    assert torch.equal(out, W[ids.long()])
    dW = torch.zeros(V, D, device=dev)
    ops().embed_bwd(ids, out, dW)
    exp = torch.zeros(V, D, device=dev).index_add_(0, ids.long(), out.float())
    assert torch.allclose(dW, exp, atol=1e-3)


def test_ppo_token_loss_matches_autograd(dev):
    """Fused PPO-RLHF token loss (policy clip + value clip) == autograd of the fp32 expression."""
    from turbol_b200.ops import reference as R_

    g = torch.Generator(device=dev).manual_seed(3)
    n = 4 * 1024 + 37
    lp = -torch.rand(n, device=dev, generator=g) * 3
    old = lp + 0.3 * torch.randn(n, device=dev, generator=g)  # ratios on both sides of the clip
    adv = torch.randn(n, device=dev, generator=g)
    v = torch.randn(n, device=dev, generator=g)
    old_v = v + 0.4 * torch.randn(n, device=dev, generator=g)
    ret = torch.randn(n, device=dev, generator=g)
    norm = 1.0 / n
    loss, dlp_ref, dv_ref, st_ref = R_.ppo_token_loss(lp, old, adv, v, old_v, ret, 0.2, 0.2, 0.1, norm)
    dlp, dv = torch.empty_like(lp), torch.empty_like(v)
    stats = torch.zeros(4, device=dev)
    ops().ppo_token_loss(lp, old, adv, v, old_v, ret, dlp, dv, stats, 0.2, 0.2, 0.1, norm)
    assert torch.allclose(dlp, dlp_ref, atol=1e-7, rtol=1e-4)
    assert torch.allclose(dv, dv_ref, atol=1e-7, rtol=1e-4)
    assert torch.allclose(stats, st_ref, rtol=1e-4, atol=1e-5), (stats, st_ref)
    assert abs(float(stats[0] + 0.1 * stats[1]) - float(loss)) < 1e-4
