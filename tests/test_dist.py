"""DistributedTrainer (reference API + collectives + mesh) on gloo CPU ranks."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

import turbol_b200 as turbol
from turbol_b200.parallel.dist import DistributedConfig, DistributedTrainer, build_mesh


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_world_one_is_a_noop():
    tr = turbol.DistributedTrainer(turbol.DistributedConfig())
    assert not tr.all_reduce(torch.ones(3)).ok()  # not initialized yet
    assert tr.initialize().ok()
    t = torch.ones(3)
    assert tr.all_reduce(t, "mean").ok() and torch.equal(t, torch.ones(3))
    assert tr.broadcast(t, 0).ok()
    assert tr.get_rank() == 0 and tr.get_world_size() == 1
    assert tr.shutdown().ok()


def test_bad_config_and_op():
    assert not DistributedTrainer(DistributedConfig(rank=3, world_size=2)).initialize().ok()
    tr = DistributedTrainer(DistributedConfig())
    tr.initialize()
    assert tr.all_reduce(torch.ones(1), "median").code() == int(turbol.turbol_core.StatusCode.kInvalidArgument)


def test_mesh_layout_without_groups():
    m = build_mesh(8, 5, tp=2, pp=2)  # no process group: coordinates only
    assert (m.tp, m.dp, m.pp) == (2, 2, 2)
    assert (m.tp_rank, m.dp_rank, m.pp_rank) == (1, 0, 1)
    with pytest.raises(ValueError):
        build_mesh(6, 0, tp=4)


def _worker(rank, world, port, q):
    try:
        tr = DistributedTrainer(DistributedConfig(rank=rank, world_size=world, master_port=port, timeout_s=60,
                                                  tp_size=2))
        assert tr.initialize().ok()
        t = torch.full((4,), float(rank + 1))
        assert tr.all_reduce(t, "sum").ok()
        assert torch.equal(t, torch.full((4,), float(sum(range(1, world + 1)))))
        t = torch.full((4,), float(rank + 1))
        assert tr.all_reduce(t, "mean").ok()
        assert torch.allclose(t, torch.full((4,), (world + 1) / 2))
        b = torch.full((3,), float(rank))
        assert tr.broadcast(b, 1).ok() and torch.equal(b, torch.ones(3))
        # core Tensor in, zero-copy
        ct = turbol.from_torch(torch.full((2,), float(rank)))
        assert tr.all_reduce(ct, "max").ok() and torch.equal(ct.torch(), torch.full((2,), world - 1.0))
        g = torch.empty(world * 2)
        assert tr.all_gather(g, torch.full((2,), float(rank))).ok()
        assert torch.equal(g, torch.arange(world).float().repeat_interleave(2))
        rs = torch.empty(2)
        assert tr.reduce_scatter(rs, torch.arange(world * 2).float()).ok()
        assert torch.equal(rs, world * torch.arange(rank * 2, rank * 2 + 2).float())
        if rank == 0:
            assert tr.send(torch.tensor([7.0, 8.0]), 1).ok()
        elif rank == 1:
            r = torch.empty(2)
            assert tr.recv(r, 0).ok() and torch.equal(r, torch.tensor([7.0, 8.0]))
        assert tr.barrier().ok()
        # tp groups of 2: sum within the pair
        m = tr.mesh
        x = torch.tensor([float(rank)])
        assert tr.all_reduce(x, "sum", group=m.tp_group).ok()
        pair = rank // 2 * 2
        assert x.item() == pair + pair + 1
        assert tr.shutdown().ok()
        q.put((rank, "ok"))
    except BaseException as e:  # reported to the parent
        q.put((rank, repr(e)))


def test_gloo_collectives_world4():
    world, port = 4, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res


def _lonely(port, q):
    tr = DistributedTrainer(DistributedConfig(rank=0, world_size=2, master_port=port, timeout_s=3))
    st = tr.initialize()  # the other rank never joins
    q.put((st.ok(), st.code()))


def test_rendezvous_timeout_is_a_status():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_port(), q))
    p.start()
    ok, code = q.get(timeout=120)
    p.join(timeout=30)
    assert not ok
