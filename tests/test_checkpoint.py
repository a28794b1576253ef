"""Checkpoint format and bit-identical resume (CPU PPO trainer)."""
import os

import pytest
import torch

import turbol_b200 as turbol
from turbol_b200.rl.ppo import PPOConfig, PPOTrainer
from turbol_b200.utils.checkpoint import latest_step, list_steps, load_checkpoint, read_config, save_checkpoint


def _cfg():
    return PPOConfig(num_envs=16, rollout_steps=8, minibatch_size=32, hidden=(16, 16), seed=3)


@pytest.mark.parametrize("background", [False, True])
def test_save_load_resume_bit_identical(tmp_path, background):
    a = PPOTrainer(_cfg(), device="cpu")
    a.train_iteration()
    h = turbol.save_checkpoint(str(tmp_path), 1, a, background=background)
    a.train_iteration()  # continue while (possibly) saving
    h.wait()
    want = a.flat.clone()
    files = sorted(os.listdir(tmp_path / "step_1"))
    assert {"policy.pt", "optim.pt", "trainer.pt", "config.cfg", "COMPLETE"} <= set(files), files
    cfg = read_config(str(tmp_path / "step_1" / "config.cfg"))
    assert cfg["num_envs"] == "16" and cfg["hidden"] == "16,16"
    # the native Config reads the same file
    c = turbol.Config()
    assert c.load(str(tmp_path / "step_1" / "config.cfg")).ok()
    assert c.get_int("rollout_steps", 0) == 8
    b = PPOTrainer(_cfg(), device="cpu")
    st = turbol.load_checkpoint(str(tmp_path), trainer=b)
    assert st["step"] == 1
    b.train_iteration()
    assert torch.equal(b.flat, want)


def test_latest_ignores_incomplete_and_config_mismatch(tmp_path):
    a = PPOTrainer(_cfg(), device="cpu")
    save_checkpoint(str(tmp_path), 5, a)
    save_checkpoint(str(tmp_path), 7, a)
    os.makedirs(tmp_path / "step_9")  # interrupted save: no COMPLETE marker
    assert list_steps(str(tmp_path)) == [5, 7] and latest_step(str(tmp_path)) == 7
    other = _cfg()
    other.lr = 1.0
    with pytest.raises(ValueError):
        load_checkpoint(str(tmp_path), config=other)
    assert load_checkpoint(str(tmp_path), config=other, strict_config=False)["step"] == 7
    save_checkpoint(str(tmp_path), 8, a, keep_last=2)
    assert list_steps(str(tmp_path)) == [7, 8]
    with pytest.raises(FileNotFoundError):
        load_checkpoint(str(tmp_path / "nothing"))
