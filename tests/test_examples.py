"""The example entry points run end to end (short runs)."""
import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "examples"))


def test_ppo_example_cpu(tmp_path):
    import ppo_example

    tr = ppo_example.main(["--device", "cpu", "--num-updates", "4", "--num-envs", "16", "--rollout-steps", "16",
                           "--batch-size", "64", "--print-every", "2", "--log-dir", str(tmp_path / "logs"),
                           "--checkpoint-dir", str(tmp_path / "ck"), "--checkpoint-every", "2"])
    assert tr.iteration == 4
    assert os.path.exists(tmp_path / "logs" / "trace.json")
    assert any(f.startswith("events.out.tfevents") for f in os.listdir(tmp_path / "logs"))
    assert sorted(os.listdir(tmp_path / "ck")) == ["step_2", "step_4"]
    tr2 = ppo_example.main(["--device", "cpu", "--num-updates", "5", "--num-envs", "16", "--rollout-steps", "16",
                            "--batch-size", "64", "--print-every", "5", "--log-dir", str(tmp_path / "logs2"),
                            "--checkpoint-dir", str(tmp_path / "ck"), "--resume"])
    assert tr2.iteration == 5


@pytest.mark.gpu
def test_ppo_example_gpu(tmp_path, dev):
    import ppo_example

    # the default fp32 compute (the 256-env workload's precision) ...
    tr = ppo_example.main(["--device", "cuda:0", "--num-updates", "3", "--num-envs", "1024", "--rollout-steps", "16",
                           "--batch-size", "4096", "--print-every", "1", "--log-dir", str(tmp_path / "fp32")])
    assert tr.iteration == 3 and not tr.fused
    # ... and bf16, which runs the fused tensor-core MLP
    tr = ppo_example.main(["--device", "cuda:0", "--num-updates", "3", "--num-envs", "1024", "--rollout-steps", "16",
                           "--batch-size", "4096", "--print-every", "1", "--log-dir", str(tmp_path / "bf16"),
                           "--dtype", "bf16"])
    assert tr.iteration == 3 and tr.fused


@pytest.mark.gpu
def test_grpo_example_gpu(tmp_path, dev):
    import grpo_example

    tr = grpo_example.main(["--num-prompts", "2", "--group-size", "4", "--prompt-len", "16", "--max-tokens", "16",
                            "--num-steps", "2", "--print-every", "1", "--micro-batch", "4", "--log-dir", str(tmp_path)])
    assert tr.step_count == 2
