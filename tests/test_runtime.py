"""Runtime services: Dataset + ByteTokenizer, TcpStore (with deadlines),
PipelineSchedule, KVBlockManager, CoreEngine."""
import json
import multiprocessing as mp
import threading
import time

import pytest
import torch

import turbol_b200 as turbol


def test_tokenizer_roundtrip():
    tok = turbol.ByteTokenizer()
    ids = tok.encode("héllo.", True, True)
    assert ids[0] == tok.bos_id and ids[-1] == tok.eos_id
    assert tok.decode(ids) == "héllo."
    assert tok.vocab_size() == 259


def test_dataset_parse_and_batches(tmp_path):
    p = tmp_path / "d.jsonl"
    rows = [{"prompt": f"q{i} \"quoted\" \\u00e9", "chosen": f"a{i}.", "rejected": "no", "meta": {"x": [1, 2]}}
            for i in range(10)]
    with open(p, "w") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")
        f.write("\n")
    s = turbol.Dataset.parse_line(json.dumps(rows[3]))
    assert s.prompt == rows[3]["prompt"] and s.chosen == "a3." and s.rejected == "no"
    cfg = turbol.DatasetConfig()
    cfg.data_paths = [str(p)]
    cfg.batch_size = 4
    cfg.max_seq_length = 64
    cfg.seed = 1
    ds = turbol.Dataset(cfg)
    assert ds.initialize().ok()
    assert ds.size() == 10
    seen = []
    while ds.has_next():
        b = ds.next_batch()
        ids = b.input_ids.torch()
        assert ids.shape[1] == 64
        seen += b.sample_indices
        m = b.attention_mask.torch()
        lab = b.labels.torch()
        pl = b.prompt_lens.torch()
        assert torch.all((lab[:, : int(pl.min())] == -100))
        assert torch.all(m.sum(1) > pl)
    assert sorted(seen) == list(range(10)) and seen != list(range(10))
    ds.reset()
    assert ds.has_next()


def test_tcp_store_threads_and_timeout():
    srv = turbol.TcpStore("127.0.0.1", 0, True, 5000)
    port = srv.port()
    cli = turbol.TcpStore("127.0.0.1", port, False, 5000)
    srv.set("k", b"v1")
    assert cli.get("k") == b"v1"
    assert cli.add("ctr", 3) == 3 and srv.add("ctr", 4) == 7
    t0 = time.time()
    with pytest.raises(RuntimeError, match="Timeout"):
        cli.get("missing", 300)
    assert time.time() - t0 < 3
    res = []

    def waiter():
        res.append(cli.get("late", 3000))

    th = threading.Thread(target=waiter)
    th.start()
    time.sleep(0.2)
    srv.set("late", b"x")
    th.join(5)
    assert res == [b"x"]


def _store_rank(port, rank, world, q):
    import turbol_b200 as tb

    s = tb.TcpStore("127.0.0.1", port, False, 10000)
    s.set(f"r{rank}", str(rank).encode())
    s.barrier("b", world, 10000)
    q.put(sorted(int(s.get(f"r{i}")) for i in range(world)))


def test_tcp_store_multiprocess_barrier_and_missing_rank():
    srv = turbol.TcpStore("127.0.0.1", 0, True, 10000)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_store_rank, args=(srv.port(), r, 3, q)) for r in range(3)]
    for p in ps:
        p.start()
    got = [q.get(timeout=60) for _ in ps]
    for p in ps:
        p.join(30)
    assert all(g == [0, 1, 2] for g in got)
    # a rank that never joins: the barrier ends with a timeout, not a hang
    c = turbol.TcpStore("127.0.0.1", srv.port(), False, 2000)
    t0 = time.time()
    with pytest.raises(RuntimeError, match="Timeout"):
        c.barrier("never", 2, 500)
    assert time.time() - t0 < 5


@pytest.mark.parametrize("P,M", [(4, 8), (2, 3), (4, 2), (1, 5)])
def test_1f1b_schedule(P, M):
    for s in range(P):
        ops = turbol.PipelineSchedule.one_f_one_b(P, s, M)
        assert [m for k, m in ops if k == "F"] == list(range(M))
        assert [m for k, m in ops if k == "B"] == list(range(M))
        # every backward comes after its forward
        pos = {(k, m): i for i, (k, m) in enumerate(ops)}
        assert all(pos[("B", m)] > pos[("F", m)] for m in range(M))
        assert turbol.PipelineSchedule.peak_activations(ops) == min(P - s, M)
    g = turbol.PipelineSchedule.gpipe(P, 0, M)
    assert turbol.PipelineSchedule.peak_activations(g) == M


def test_kv_block_manager():
    kv = turbol.KVBlockManager(8, 16)
    assert kv.allocate(1, 20).ok() and len(kv.block_table(1)) == 2
    for _ in range(12):
        assert kv.append_token(1).ok()
    assert kv.seq_len(1) == 32 and len(kv.block_table(1)) == 2
    assert kv.append_token(1).ok() and len(kv.block_table(1)) == 3
    assert not kv.allocate(2, 16 * 6).ok()  # 5 free blocks
    assert kv.allocate(2, 16 * 5).ok() and kv.num_free() == 0
    assert not kv.append_token(2).ok()
    assert kv.free(1).ok() and kv.num_free() == 3
    assert set(kv.block_table(2)).isdisjoint({-1})


def test_core_engine():
    ce = turbol.CoreEngine.instance()
    assert ce.initialize(0, 2).ok()
    ce.register_module("env")
    assert ce.has_module("env") and "env" in ce.list_modules()
    assert ce.synchronize().ok()
    assert ce.shutdown().ok()
