"""Filtered sampler (temperature, top-k, top-p, end-of-sequence stop) against
plain fp32 PyTorch: the kept set of a row (sorted softmax), empirical
frequencies of the truncated, renormalized distribution, log-probs under the
full tempered softmax, and the done / length bookkeeping of the EOS stop."""
import pytest
import torch

from turbol_b200._native import ops

pytestmark = pytest.mark.gpu


def bf(x):
    return x.to(torch.bfloat16)


def kept_mask(row: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    """fp32 oracle of the kept set: top-k (ties at the k-th value kept), then the
    smallest prefix of the remaining tokens, by descending probability, whose mass
    reaches top_p of theirs (ties at the boundary value kept)."""
    z = row.float() / temperature
    keep = torch.ones_like(z, dtype=torch.bool)
    if 0 < top_k < z.numel():
        kth = torch.topk(z, top_k).values[-1]
        keep &= z >= kth
    if top_p < 1.0:
        p = torch.softmax(torch.where(keep, z, torch.full_like(z, -float("inf"))), -1).double()
        vals, _ = torch.sort(p, descending=True)
        cum = torch.cumsum(vals, 0)
        idx = int(torch.searchsorted(cum, torch.tensor(top_p, dtype=torch.float64, device=cum.device) - 1e-12))
        thr = vals[min(idx, vals.numel() - 1)]
        keep &= p >= thr
    return keep


def sample(logits, t, k, p, seed, step=0, **kw):
    B = logits.shape[0]
    tok = torch.empty(B, device=logits.device, dtype=torch.int32)
    lp = torch.empty(B, device=logits.device)
    ops().sample_filtered(logits, t, k, p, seed, None, step, tok, lp, **kw)
    return tok, lp


@pytest.mark.parametrize("top_k,top_p", [(50, 1.0), (-1, 0.9), (200, 0.8), (1, 1.0)])
def test_tokens_stay_in_the_kept_set(dev, top_k, top_p):
    B, V = 64, 151936
    logits = bf(torch.randn(B, V, device=dev) * 2.5)
    tok, lp = sample(logits, 0.8, top_k, top_p, seed=5)
    for b in range(B):
        keep = kept_mask(logits[b], 0.8, top_k, min(1.0, top_p + 1e-4) if top_p < 1.0 else 1.0)  # boundary slack
        assert keep[tok[b].long()], (b, int(tok[b]))
    full = torch.log_softmax(logits.float() / 0.8, -1).gather(1, tok.long()[:, None])[:, 0]
    assert torch.allclose(lp, full, atol=2e-3)


@pytest.mark.parametrize("top_k,top_p", [(3, 1.0), (-1, 0.7), (4, 0.8)])
def test_frequencies_follow_the_truncated_distribution(dev, top_k, top_p):
    base = torch.tensor([2.0, 1.5, 1.0, 0.5, 0.0, -0.5, -1.0, -3.0] * 4)  # V = 32 (vector path)
    n = 32768
    logits = bf(base.repeat(n, 1).to(dev))
    tok, _ = sample(logits, 1.0, top_k, top_p, seed=11, step=3)
    keep = kept_mask(logits[0], 1.0, top_k, top_p)
    z = torch.where(keep, logits[0].float(), torch.full_like(logits[0].float(), -float("inf")))
    want = torch.softmax(z, -1)
    freq = torch.bincount(tok.long(), minlength=32).float() / n
    assert (freq - want).abs().max().item() < 0.015
    assert freq[~keep].sum().item() == 0.0


def test_greedy_and_odd_width_rows(dev):
    B, V = 9, 1001  # V % 8 != 0: scalar path
    logits = bf(torch.randn(B, V, device=dev) * 3)
    tok, _ = sample(logits, 0.0, 10, 0.5, seed=1)
    assert torch.equal(tok.long(), logits.float().argmax(-1))
    tok, _ = sample(logits, 1.0, 5, 1.0, seed=2)
    for b in range(B):
        assert kept_mask(logits[b], 1.0, 5, 1.0)[tok[b].long()]


def test_eos_stop_sets_done_and_lengths(dev):
    B, V, steps, eos, pad = 16, 512, 6, 7, 0
    done = torch.zeros(B, device=dev, dtype=torch.uint8)
    lengths = torch.full((B,), steps, device=dev, dtype=torch.int32)
    n_done = torch.zeros(1, device=dev, dtype=torch.int32)
    tok_mat = torch.full((B, steps), -5, device=dev, dtype=torch.int32)
    lp_mat = torch.zeros(B, steps, device=dev)
    step_t = torch.zeros(1, device=dev, dtype=torch.int64)
    tok = torch.empty(B, device=dev, dtype=torch.int32)
    for s in range(steps):
        logits = torch.full((B, V), -4.0, device=dev)
        # row b emits eos at step b (rows >= steps never do)
        for b in range(B):
            logits[b, eos if b == s else (100 + b)] = 20.0
        ops().sample_filtered(bf(logits), 1.0, -1, 1.0, 3, step_t, 0, tok, None, tok_mat, lp_mat, eos_id=eos,
                              pad_id=pad, done=done, lengths=lengths, n_done=n_done)
        step_t += 1
    torch.cuda.synchronize()
    for b in range(B):
        if b < steps:
            assert done[b] == 1 and lengths[b] == b + 1
            assert tok_mat[b, b] == eos and bool((tok_mat[b, b + 1:] == pad).all())
            assert bool((lp_mat[b, b + 1:] == 0).all())
            assert bool((tok_mat[b, :b] == 100 + b).all())
        else:
            assert done[b] == 0 and lengths[b] == steps and bool((tok_mat[b] == 100 + b).all())
    assert int(n_done) == steps


def test_generator_eos_and_filters(dev):
    """The decode loop stops when every sequence has emitted eos; filters run in the captured step."""
    from turbol_b200.models.llm import DecoderLM, LMConfig
    from turbol_b200.rl.rollout import LLMGenerator

    cfg = LMConfig.tiny(vocab=512, n_layers=2)
    m = DecoderLM(cfg, dev, seed=1, master=False)
    gen = LLMGenerator(m, 32, 128, seed=3)
    prompts = torch.randint(0, cfg.vocab, (4, 16), dtype=torch.int32)
    seqs, lp = gen.generate(prompts, 2, 24, 1.0, top_k=20, top_p=0.9)
    assert seqs.shape == (8, 40) and torch.isfinite(lp).all()
    # greedy with top-k: deterministic and equal to the plain greedy sampler
    a, _ = gen.generate(prompts, 1, 12, 0.0, top_k=5)
    b, _ = gen.generate(prompts, 1, 12, 0.0)
    assert torch.equal(a, b)
    # eos = the greedy second token of each sequence: every row stops at step 1
    g, _ = gen.generate(prompts, 1, 12, 0.0)
    eos_tokens = g[:, 17]
    eos = int(eos_tokens[0])
    s, lp = gen.generate(prompts, 1, 12, 0.0, eos_id=eos, pad_id=0)
    L = gen.last_lengths.cpu()
    for r in range(4):
        row = g[r, 16:].tolist()
        n = row.index(eos) + 1 if eos in row else 12
        assert int(L[r]) == n
        assert s[r, 16:16 + n].tolist() == row[:n] and all(t == 0 for t in s[r, 16 + n:].tolist())
