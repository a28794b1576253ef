"""Activation recompute in a pipeline stage (one GPU, one stage): the 1F1B
pass with recomputation gives the gradients of the pass that keeps every
activation, and holds less memory between a micro-batch's forward and its
backward.  The multi-stage case runs in tests/pp_worker.py."""
import pytest
import torch

from turbol_b200._native import ops
from turbol_b200.models.llm import LMConfig
from turbol_b200.parallel import pipeline as pp

pytestmark = pytest.mark.gpu


def _loss_grad(model, x, ids):
    o = ops()
    N = x.shape[0]
    rstd = torch.empty(N, device=x.device)
    hf = model.final_norm(x, rstd)
    logits = model.logits(hf)
    tgt = torch.roll(ids.reshape(-1), -1).contiguous()
    dlp = torch.full((N,), -1e-3, device=x.device)
    o.logprob(logits, tgt, None, dlp)
    dh = torch.empty_like(hf)
    o.gemm(logits, model.head_weight(), dh, False, True)
    o.gemm(logits, hf, model.head_grad(), True, True, accumulate=True, split_k=1)
    dx = torch.empty_like(x)
    o.rmsnorm_bwd(dh, x, model.f32["norm"], rstd, dx, None, model.g["norm"])
    return dx


def test_recompute_matches_and_saves_memory(dev):
    cfg = LMConfig.tiny(n_layers=4)
    cfg.tie_embeddings = False
    st = pp.PipelineStage(cfg, 0, 1, dev, seed=3)
    mb, T, M = 4, 256, 4
    ids = torch.randint(0, cfg.vocab, (mb * M, T), generator=torch.Generator().manual_seed(1)).to(dev, torch.int32)
    pp.set_micro_geometry(mb, T, torch.arange(T, device=dev, dtype=torch.int32).repeat(mb))
    held = {}

    def run(recompute):
        st.zero_grad()
        torch.cuda.synchronize()
        held[recompute] = []

        def loss(i, x):
            # memory alive when the last stage starts the backward of micro-batch i
            torch.cuda.synchronize()
            held[recompute].append(torch.cuda.memory_allocated(dev))
            return _loss_grad(st.model, x, ids[i * mb:(i + 1) * mb])

        pp.run_1f1b(st, [0], M, mb * T, lambda i: st.model.embed(ids[i * mb:(i + 1) * mb]), loss,
                    lambda i, dx: st.model.embed_backward(ids[i * mb:(i + 1) * mb], dx), recompute=recompute)
        torch.cuda.synchronize()
        return st.model.grad.clone()

    g_keep = run(False)
    g_re = run(True)
    rel = (g_re - g_keep).abs().max().item() / (g_keep.abs().max().item() + 1e-12)
    assert rel < 1e-5, rel
    # the saved activations of a micro-batch (every layer's inputs, attention
    # statistics, MLP activations) are gone with recompute
    assert max(held[True]) < max(held[False]), (held[True], held[False])
