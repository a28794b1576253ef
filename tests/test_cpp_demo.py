"""The native C++ demo (examples/cpp) builds against the compiled core and
runs on CPU through the C++ API alone."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEMO = os.path.join(ROOT, "examples", "cpp")


@pytest.mark.skipif(shutil.which("make") is None or shutil.which(os.environ.get("CXX", "g++")) is None,
                    reason="no C++ toolchain")
def test_cpp_demo_builds_and_runs():
    b = subprocess.run(["make", "-C", DEMO], capture_output=True, text=True, timeout=600)
    assert b.returncode == 0, b.stdout[-2000:] + b.stderr[-2000:]
    r = subprocess.run([os.path.join(DEMO, "turbol_demo"), "cpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    out = r.stdout
    assert "200 steps x 1024 envs" in out and "sampled 256 rows" in out and "demo finished" in out
    assert "rank 0 of 1, all-reduce(mean) ok" in out
