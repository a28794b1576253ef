"""Race and memory checks of the host core under the compiler's sanitizers
(AddressSanitizer + UndefinedBehaviorSanitizer in one build, ThreadSanitizer in
another; tests/native/host_sanitize.cpp drives the profiler from several
threads, the TCP store with concurrent clients, the KV block allocator, the
file formats, and the CPU trainer's host engines from two threads).
Device-side checking is done by the kernels' own error words; this covers the
host runtime around them."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NATIVE = os.path.join(ROOT, "tests", "native")
OUT = os.path.join(ROOT, "build", "sanitize")
SANCXX = os.environ.get("SANCXX", "/usr/bin/g++")


def _have_runtime(name: str) -> bool:
    if not shutil.which(SANCXX) or not shutil.which("make"):
        return False
    r = subprocess.run([SANCXX, f"-print-file-name=lib{name}.so"], capture_output=True, text=True)
    return r.returncode == 0 and os.path.isabs(r.stdout.strip())


@pytest.mark.parametrize("kind,runtime,env", [
    ("asan", "asan", {"ASAN_OPTIONS": "detect_leaks=1:detect_odr_violation=0",
                      "UBSAN_OPTIONS": "print_stacktrace=1:halt_on_error=1"}),
    ("tsan", "tsan", {"TSAN_OPTIONS": "halt_on_error=1:second_deadlock_stack=1"}),
])
@pytest.mark.timeout(2700)  # build (up to 900 s) + instrumented run (up to 1500 s) on a slow, shared machine
def test_host_core_under_sanitizer(kind, runtime, env):
    if not _have_runtime(runtime):
        pytest.skip(f"no lib{runtime} for {SANCXX}")
    b = subprocess.run(["make", "-s", "-j8", "-C", NATIVE, kind, f"SANCXX={SANCXX}", f"OUT={OUT}"],
                       capture_output=True, text=True, timeout=900)
    assert b.returncode == 0, b.stdout[-3000:] + b.stderr[-3000:]
    with tempfile.TemporaryDirectory() as d:
        r = subprocess.run([os.path.join(OUT, f"host_sanitize_{kind}"), d], capture_output=True, text=True,
                           timeout=1500, env=dict(os.environ, **env))
    report = r.stdout[-4000:] + r.stderr[-4000:]
    assert r.returncode == 0 and "HOST_SANITIZE_OK" in r.stdout, report
    for marker in ("ERROR: AddressSanitizer", "runtime error:", "WARNING: ThreadSanitizer"):
        assert marker not in r.stderr, report
