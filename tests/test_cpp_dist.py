"""The C++ distributed runtime (turbol_core.dist): single-process behaviour on
any machine with the CUDA build, and the two-GPU worker (NCCL collectives,
DistributedTrainer, 1F1B PipelineTrainer) where two GPUs exist."""
import os
import socket
import subprocess
import sys

import pytest
import torch

import turbol_b200

HERE = os.path.dirname(os.path.abspath(__file__))
D = getattr(turbol_b200.turbol_core, "dist", None)
needs_dist = pytest.mark.skipif(D is None, reason="CPU-only build: no NCCL runtime")


@needs_dist
def test_world_of_one_and_bad_configs():
    cfg = D.DistributedConfig()
    tr = D.DistributedTrainer(cfg)
    assert not tr.all_reduce(torch.ones(3), "sum").ok()  # not initialized
    assert tr.initialize().ok() and tr.get_world_size() == 1 and tr.get_rank() == 0
    t = torch.ones(3)
    assert tr.all_reduce(t, "sum").ok() and torch.equal(t, torch.ones(3))  # a group of one
    assert tr.all_reduce(t, "median").code() == int(turbol_b200.StatusCode.kInvalidArgument)
    bad = D.DistributedConfig()
    bad.rank, bad.world_size = 3, 2
    assert not D.DistributedTrainer(bad).initialize().ok()
    comm = D.NcclCommunicator()
    assert not comm.all_reduce(torch.ones(1), "sum").ok()  # not initialized


@needs_dist
def test_pipeline_trainer_one_stage_order_and_recompute():
    """One stage (no communicator needed): 1F1B degenerates to F0 B0 F1 B1 ...,
    the loss is the micro-batch mean and recompute runs before each backward."""
    M = 4
    cfg = D.PipelineConfig()
    cfg.num_microbatches, cfg.hidden_size, cfg.microbatch_seq_len = M, 8, 4
    cfg.activation_checkpointing = True
    calls = []
    pt = D.PipelineTrainer(cfg)
    st = pt.initialize(None, input=lambda i: torch.full((4, 8), float(i)),
                       forward=lambda i, x: (calls.append(("F", i)), x * 2)[1],
                       loss=lambda i, y: (float(y.sum()), torch.ones_like(y)),
                       backward=lambda i, d: (calls.append(("B", i)), d)[1],
                       recompute=lambda i, x: calls.append(("R", i)), dtype="float32")
    assert st.ok(), st
    st, loss = pt.training_step()
    assert st.ok(), st
    assert pt.last_order() == [f"{k}{i}" for i in range(M) for k in "FB"]
    assert calls == [(k, i) for i in range(M) for k in "FRB"]
    assert abs(loss - sum(64.0 * i for i in range(M)) / M) < 1e-5
    cfg2 = D.PipelineConfig()
    cfg2.hidden_size = 8
    cfg2.activation_checkpointing = True  # without a recompute function
    assert not D.PipelineTrainer(cfg2).initialize(None, input=lambda i: None, forward=lambda i, x: x,
                                                  loss=lambda i, y: (0.0, y), backward=lambda i, d: d).ok()


@pytest.mark.gpu
@pytest.mark.multigpu
@needs_dist
def test_cpp_distributed_runtime_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TB_CPP_PORT=str(port))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29547", os.path.join(HERE, "cpp_dist_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0 and "CPP_DIST_WORKER_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
