"""Profiler, TensorBoard (TFRecord) and Prometheus writers.  Covers the
reference's ProfilerTest cases (turbol_vllm/tests/test_profiler_reward.cpp:26-110)
plus the exports those tests never called (where the reference deadlocks)."""
import json
import os
import struct
import threading
import time

import numpy as np
import pytest

import turbol_b200 as turbol


def spin(ms):
    t = time.perf_counter()
    while (time.perf_counter() - t) * 1e3 < ms:
        pass


def test_spans_nesting_and_ids():
    p = turbol.Profiler(turbol.ProfilerConfig())
    assert not p.is_enabled()
    p.enable()
    outer = p.begin_span("outer")
    inner = p.begin_span("inner")
    spin(2)
    # end out of order: ids decide which span ends
    p.end_span(outer)
    p.end_span(inner)
    spans = {s.name: s for s in p.get_all_spans()}
    assert spans["inner"].parent == spans["outer"].id
    assert spans["inner"].duration_ns() >= 1_000_000
    with p.span("guarded"):
        spin(1)
    with turbol.ProfilerGuard(p, "guard2", "io", -1):
        spin(1)
    stats = {s.name: s for s in p.get_stats()}
    assert stats["guarded"].count == 1 and stats["guarded"].total_ns >= 900_000
    assert stats["guard2"].count == 1
    p.mark("point")
    p.disable()
    assert p.begin_span("ignored").id == 0


def test_exports_do_not_deadlock(tmp_path):
    p = turbol.Profiler(turbol.ProfilerConfig())
    p.enable()
    for i in range(3):
        with p.span("step"):
            spin(0.2)
    p.record_comm("allreduce", 1 << 20, 0.5)
    done = []

    def run():
        assert p.export_json(str(tmp_path / "s.json")).ok()
        assert p.export_chrome_trace(str(tmp_path / "t.json")).ok()
        done.append(1)

    th = threading.Thread(target=run)
    th.start()
    th.join(timeout=10)
    assert done, "export deadlocked"
    js = json.load(open(tmp_path / "s.json"))
    assert js["stats"][0]["count"] == 3 and js["comms"][0]["bytes"] == 1 << 20
    tr = json.load(open(tmp_path / "t.json"))
    assert all(e["ph"] == "X" for e in tr) and len(tr) == 3
    assert "step" in p.summary()


def _read_records(path):
    out = []
    with open(path, "rb") as f:
        data = f.read()
    i = 0
    while i < len(data):
        (n,) = struct.unpack("<Q", data[i:i + 8])
        (hc,) = struct.unpack("<I", data[i + 8:i + 12])
        assert hc == turbol.turbol_core.masked_crc32c(data[i:i + 8])
        payload = data[i + 12:i + 12 + n]
        (pc,) = struct.unpack("<I", data[i + 12 + n:i + 16 + n])
        assert pc == turbol.turbol_core.masked_crc32c(payload)
        out.append(payload)
        i += 16 + n
    return out


def _varint(b, i):
    r, s = 0, 0
    while True:
        c = b[i]
        i += 1
        r |= (c & 0x7F) << s
        s += 7
        if c < 0x80:
            return r, i


def _fields(b):
    i, out = 0, []
    while i < len(b):
        key, i = _varint(b, i)
        f, w = key >> 3, key & 7
        if w == 0:
            v, i = _varint(b, i)
        elif w == 1:
            v = b[i:i + 8]
            i += 8
        elif w == 5:
            v = b[i:i + 4]
            i += 4
        elif w == 2:
            n, i = _varint(b, i)
            v = b[i:i + n]
            i += n
        else:
            raise AssertionError(f"bad wire type {w}")
        out.append((f, w, v))
    return out


def test_crc32c_known_vector():
    # RFC 3720 test vector: 32 bytes of zeros -> 0x8A9136AA
    assert turbol.turbol_core.crc32c(b"\x00" * 32) == 0x8A9136AA
    assert turbol.turbol_core.crc32c(b"123456789") == 0xE3069283


def test_tensorboard_event_file_is_valid(tmp_path):
    w = turbol.TensorBoardWriter(str(tmp_path))
    w.add_scalar("train/loss", 0.5, 3)
    w.add_histogram("w", np.arange(10, dtype=np.float32), 4)
    w.add_text("note", "hello", 5)
    w.flush()
    recs = _read_records(w.path())
    assert len(recs) == 4
    first = dict((f, v) for f, _, v in _fields(recs[0]))
    assert first[3] == b"brain.Event:2"
    ev = _fields(recs[1])
    d = {f: (wt, v) for f, wt, v in ev}
    assert d[1][0] == 1 and isinstance(struct.unpack("<d", d[1][1])[0], float)  # wall_time double
    assert d[2] == (0, 3)  # step varint
    summ = _fields(d[5][1])
    val = dict((f, v) for f, _, v in _fields(summ[0][2]))
    assert val[1] == b"train/loss" and abs(struct.unpack("<f", val[2])[0] - 0.5) < 1e-7
    hv = dict((f, v) for f, _, v in _fields(_fields(dict((f, v) for f, _, v in _fields(recs[2]))[5])[0][2]))
    histo = dict((f, v) for f, _, v in _fields(hv[5]))
    assert struct.unpack("<d", histo[3])[0] == 10.0 and struct.unpack("<d", histo[4])[0] == 45.0


def test_prometheus_writer(tmp_path):
    p = turbol.PrometheusWriter(str(tmp_path / "m.prom"))
    lab = turbol.Labels()
    lab["rank"] = "0"
    p.write_counter("steps_total", 5, lab)
    p.write_counter("steps_total", 2, lab)
    p.write_gauge("fps", 123.5)
    p.observe_histogram("step_ms", 3.0, [1, 5, 10])
    p.observe_histogram("step_ms", 7.0, [1, 5, 10])
    assert p.flush().ok()
    text = open(tmp_path / "m.prom").read()
    assert "# TYPE steps_total counter" in text and 'steps_total{rank="0"} 7' in text
    assert "fps 123.5" in text
    assert 'step_ms_bucket{le="5"} 1' in text and 'step_ms_bucket{le="10"} 2' in text
    assert 'step_ms_bucket{le="+Inf"} 2' in text and "step_ms_count 2" in text


@pytest.mark.gpu
def test_cuda_events(dev):
    import torch

    p = turbol.Profiler(turbol.ProfilerConfig())
    p.enable()
    e = p.begin_event("mm", 0)
    a = torch.randn(2048, 2048, device=dev)
    for _ in range(10):
        a = a @ a / 2048
    p.end_event(e)
    st = {s.name: s for s in p.get_stats()}
    assert st["mm"].count == 1 and st["mm"].total_ns > 0
