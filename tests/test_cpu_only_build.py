"""The CPU-only build of the native core (TURBOL_CPU_ONLY=1): the host runtime
compiled by the C++ compiler alone, no nvcc, no CUDA headers or runtime.

The build goes to a temporary directory (never over the in-tree CUDA build);
a fresh interpreter that cannot see the repository imports it and runs the
reference's CPU-side API through it: Status codes, Tensor, Config round trip,
the linear environment and CartPole, RingBuffer, RewardEngine, Profiler and
the TensorBoard writer, the tokenizer and the KV block allocator.  The
reference's minimal tree is the same idea (turbol/CMakeLists.txt:1-34: its
core without CUDA)."""
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHECK = r'''
import sys, tempfile, os
sys.path = [p for p in sys.path if os.path.abspath(p or ".") != REPO]
sys.path.insert(0, LIB)
import numpy as np
import torch
from turbol_b200 import turbol_core as C
assert C.built_for() == "cpu", C.built_for()
assert not hasattr(C, "ops")
assert int(C.StatusCode.kUnimplemented) == 5 and int(C.StatusCode.kInternalError) == 6
assert C.get_device_count() == 0
t = C.Tensor([2, 3], "float32", "cpu")
assert t.numel() == 6 and t.device() == "CPU"
d = tempfile.mkdtemp()
c = C.Config(); c.set("lr", "0.5"); c.set("name", "x")
assert c.save(os.path.join(d, "a.cfg")).ok()
c2 = C.Config(); assert c2.load(os.path.join(d, "a.cfg")).ok() and c2.get_float("lr", 0.0) == 0.5
env = C.GPUEnvironment(8, 4, 2, "cpu")
obs, rew, done = env.step(C.Tensor([8, 2], "float32", "cpu"))
assert obs.numel() == 32 and rew.numel() == 8
cp = C.GPUEnvironment(16, 4, 2, "cpu", "cartpole", seed=3)
buf = C.RingBuffer(64, 4, 2, "cpu")
for _ in range(3):
    o, r, dn = env.step(C.Tensor([8, 2], "float32", "cpu"))
    assert buf.push_batch(o, C.Tensor([8, 2], "float32", "cpu"), r, dn).ok()
assert buf.size() == 24
so, sa, sr, sd = (C.Tensor([5, 4], "float32", "cpu"), C.Tensor([5, 2], "float32", "cpu"),
                  C.Tensor([5], "float32", "cpu"), C.Tensor([5], "bool", "cpu"))
assert buf.sample(5, so, sa, sr, sd).ok()
rc = C.RewardConfig(); rc.normalize = True
re_ = C.RewardEngine(rc); assert re_.initialize().ok()
res = re_.score_batch(["Hello world.", "abc"])
assert res.total.numel() == 2
p = C.Profiler(); p.enable()
sid = p.begin_span("x", "t"); p.end_span(sid)
assert p.export_json(os.path.join(d, "p.json")).ok()
w = C.TensorBoardWriter(d); w.add_scalar("a", 1.0, 1); w.flush()
tok = C.ByteTokenizer(); assert tok.decode(tok.encode("hi", True, True), True) == "hi"
kv = C.KVBlockManager(8, 16); assert kv.allocate(0, 40).ok() and len(kv.block_table(0)) == 3
print("CPU_ONLY_OK")
'''


@pytest.mark.skipif(shutil.which("g++") is None and shutil.which("c++") is None, reason="no C++ compiler")
def test_cpu_only_core_builds_and_runs(tmp_path):
    lib, tmp = tmp_path / "lib", tmp_path / "tmp"
    env = dict(os.environ, TURBOL_CPU_ONLY="1", MAX_JOBS=str(max(1, os.cpu_count() or 1)))
    b = subprocess.run([sys.executable, "setup.py", "build_ext", "--build-lib", str(lib), "--build-temp", str(tmp)],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=1200)
    assert b.returncode == 0, b.stdout[-3000:] + b.stderr[-3000:]
    sos = list((lib / "turbol_b200").glob("turbol_core*.so"))
    assert len(sos) == 1, sos
    # nothing of CUDA is linked in
    if shutil.which("ldd"):
        deps = subprocess.run(["ldd", str(sos[0])], capture_output=True, text=True).stdout
        assert "libcudart" not in deps and "libtorch_cuda" not in deps and "libc10_cuda" not in deps, deps
    code = f"REPO = {ROOT!r}\nLIB = {str(lib)!r}\n" + CHECK
    r = subprocess.run([sys.executable, "-c", code], cwd=str(tmp_path), capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "CPU_ONLY_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]
