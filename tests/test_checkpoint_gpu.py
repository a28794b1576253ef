"""Checkpoint / resume of the GPU trainers (one GPU): the fused PPO path
(weights in the tensor-core MLP's flat buffers, Adam on the device, device
counters) and GRPO on a small decoder.  Restoring is exact (every saved tensor
comes back bit for bit); the first step after the resume reproduces the
uninterrupted run's step to within 1 % of that step's update (the weight- and
bias-gradient reductions add in hardware order, so the last bits can differ).
The sharded layouts (tensor- and pipeline-parallel) are checked in the
two-GPU workers."""
import os

import pytest
import torch

from turbol_b200.utils.checkpoint import load_checkpoint, save_checkpoint

pytestmark = pytest.mark.gpu


def _close_update(after, before, want):
    """|after - want| <= 1 % of the step's update |want - before| (max norms)."""
    upd = (want - before).abs().max().item()
    err = (after - want).abs().max().item()
    assert upd > 0, "the step did not change the weights"
    assert err <= 1e-2 * upd, (err, upd)


def test_fused_ppo_save_and_resume(tmp_path, dev):
    from turbol_b200.rl.ppo import PPOConfig, PPOTrainer

    cfg = PPOConfig(num_envs=4096, rollout_steps=16, hidden=(256, 256), epochs=2, minibatch_size=8192,
                    compute_dtype="bf16", cuda_graphs=False, seed=5)
    a = PPOTrainer(cfg, device=dev)
    assert a.fused
    a.train_iteration()
    save_checkpoint(str(tmp_path), 1, a, background=True).wait()
    saved = {"flat": a.flat.clone(), "m": a.opt.m.clone(), "v": a.opt.v.clone(), "state": a.state.clone(),
             "iter": int(a.iter_t.item())}
    a.train_iteration()
    b = PPOTrainer(cfg, device=dev)
    st = load_checkpoint(str(tmp_path), trainer=b)
    assert st["step"] == 1 and b.iteration == 1
    assert torch.equal(b.flat, saved["flat"]) and torch.equal(b.net.shadow, saved["flat"].to(torch.bfloat16))
    assert torch.equal(b.opt.m, saved["m"]) and torch.equal(b.opt.v, saved["v"])
    assert torch.equal(b.state, saved["state"]) and int(b.iter_t.item()) == saved["iter"]
    b.train_iteration()
    torch.cuda.synchronize()
    _close_update(b.flat, saved["flat"], a.flat)


def test_grpo_save_and_resume(tmp_path, dev):
    from turbol_b200.models.llm import LMConfig
    from turbol_b200.rl.grpo import GRPOConfig, GRPOTrainer

    cfg = GRPOConfig(model=LMConfig.tiny(n_layers=2, vocab=512), num_prompts=4, group_size=4, prompt_len=32,
                     response_len=32, micro_batch=4, lr=1e-3)
    a = GRPOTrainer(cfg, dev)
    a.step()
    save_checkpoint(str(tmp_path), 1, a)
    files = set(os.listdir(tmp_path / "step_1"))
    assert {"policy.pt", "optim.pt", "trainer.pt", "config.cfg", "COMPLETE"} <= files, files
    saved = a.model.flat.clone()
    a.step()
    b = GRPOTrainer(cfg, dev)
    load_checkpoint(str(tmp_path), trainer=b)
    assert torch.equal(b.model.flat, saved) and b.step_count == 1 and b.gen.calls == a.gen.calls - 1
    assert torch.equal(b.ref.shadow, a.ref.shadow)
    b.step()
    torch.cuda.synchronize()
    _close_update(b.model.flat, saved, a.model.flat)
