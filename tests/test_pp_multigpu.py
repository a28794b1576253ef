"""Pipeline parallelism (1F1B over NCCL p2p) and PPO-RLHF on 2 GPUs (skipped with fewer)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HERE = os.path.dirname(os.path.abspath(__file__))


def test_pipeline_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "500", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29539", os.path.join(HERE, "pp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "PP_WORKER_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def _run_pp_tp(n: int, port: int):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "500", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(HERE, "pp_tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "PP_TP_WORKER_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_pipeline_tensor_parallel_two_gpus():
    """One pipeline stage of two TP ranks (the TP stage, loss head, value head and weight sync)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run_pp_tp(2, 29543)


def test_pipeline_tensor_parallel_four_gpus():
    """Two stages x two TP ranks."""
    if torch.cuda.device_count() < 4:
        pytest.skip("needs 4 GPUs")
    _run_pp_tp(4, 29547)
