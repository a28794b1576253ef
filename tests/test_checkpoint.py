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


def test_step_complete_needs_every_rank_marker(tmp_path):
    """A data-parallel save is complete only when every rank's marker is there."""
    from turbol_b200.utils.checkpoint import step_complete

    a = PPOTrainer(_cfg(), device="cpu")
    lay = {"tp": 1, "pp": 1, "dp": 2}
    save_checkpoint(str(tmp_path), 3, a, dp_rank=0, layout=lay)
    assert not step_complete(str(tmp_path / "step_3")) and latest_step(str(tmp_path)) is None
    with pytest.raises(FileNotFoundError):
        load_checkpoint(str(tmp_path), 3, dp_rank=0, layout=lay)
    save_checkpoint(str(tmp_path), 3, a, dp_rank=1, layout=lay)
    assert step_complete(str(tmp_path / "step_3")) and latest_step(str(tmp_path)) == 3
    files = set(os.listdir(tmp_path / "step_3"))
    assert {"policy.pt", "optim_dp0.pt", "optim_dp1.pt", "trainer_dp0.pt", "trainer_dp1.pt",
            "COMPLETE_dp0", "COMPLETE_dp1"} <= files, files
    # a tensor x pipeline layout names every shard and needs all of them
    lay2 = {"tp": 2, "pp": 2, "dp": 0}
    for t in range(2):
        for p in range(2):
            assert not step_complete(str(tmp_path / "step_4"))  # until the last of the four shards
            save_checkpoint(str(tmp_path), 4, a, tp_rank=t, pp_rank=p, layout=lay2)
    files = set(os.listdir(tmp_path / "step_4"))
    assert {f"policy_tp{t}_pp{p}.pt" for t in range(2) for p in range(2)} <= files, files
    assert step_complete(str(tmp_path / "step_4"))
    with pytest.raises(ValueError):  # a different layout than the save's
        load_checkpoint(str(tmp_path), 3, dp_rank=0, layout={"tp": 1, "pp": 1, "dp": 4})
    # keep_last never counts or removes a step that is still incomplete
    save_checkpoint(str(tmp_path), 6, a, dp_rank=0, layout=lay)  # rank 1 not done yet
    save_checkpoint(str(tmp_path), 5, a, keep_last=1)
    assert list_steps(str(tmp_path)) == [5] and os.path.isdir(tmp_path / "step_6")


def _dp_ckpt_worker(rank, world, port, path, q):
    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        cfg = _cfg()
        a = PPOTrainer(cfg, device="cpu", rank=rank, dp="nccl")  # gradient all-reduce over the group (gloo here)
        a.train_iteration()
        save_checkpoint(path, 1, a)          # ranks and layout come from a.checkpoint_ranks()
        dist.barrier()
        a.train_iteration()
        want = (a.flat.clone(), a.state.clone())
        b = PPOTrainer(cfg, device="cpu", rank=rank, dp="nccl")
        st = load_checkpoint(path, trainer=b)  # this rank's own environments and RNG
        b.train_iteration()
        ok = st["step"] == 1 and torch.equal(b.flat, want[0]) and torch.equal(b.state, want[1])
        q.put((rank, bool(ok), ""))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, False, repr(e)))


def test_data_parallel_save_and_resume_per_rank(tmp_path):
    """Two gloo ranks save their own shards and resume bit-identically."""
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_dp_ckpt_worker, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
    files = set(os.listdir(tmp_path / "step_1"))
    assert {"trainer_dp0.pt", "trainer_dp1.pt", "COMPLETE_dp0", "COMPLETE_dp1"} <= files, files
