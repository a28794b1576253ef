#!/usr/bin/env python
"""Profiler overhead per span (host side; no GPU needed).

  python benchmarks/benchmark_profiler.py [--spans 200000]

Times begin_span/end_span pairs and the `with profiler.span(...)` context
manager through the Python API, with the profiler enabled (spans recorded and
aggregated) and disabled (the early-out path), plus the cost of exporting the
recorded spans as a Chrome trace and as JSON statistics.  The reference's
Profiler (turbol_vllm/src/profiler/profiler.cpp:46-83) has the same span API;
its ExportJSON locks its mutex twice and cannot return.
"""
import argparse
import json
import os
import sys
import tempfile
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import turbol_b200 as turbol  # noqa: E402


def per_op_ns(fn, n):
    t0 = time.perf_counter_ns()
    fn(n)
    return (time.perf_counter_ns() - t0) / n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--spans", type=int, default=200000)
    a = ap.parse_args()
    cfg = turbol.ProfilerConfig()
    cfg.enable_cuda_timing = False
    prof = turbol.Profiler(cfg)

    def pairs(n):
        for i in range(n):
            prof.end_span(prof.begin_span("step"))

    def guards(n):
        for i in range(n):
            with prof.span("step"):
                pass

    out = {"benchmark": "profiler_span_overhead", "spans": a.spans}
    prof.disable()
    out["disabled_pair_ns"] = per_op_ns(pairs, a.spans)
    prof.enable()
    out["enabled_pair_ns"] = per_op_ns(pairs, a.spans)
    prof.clear()
    out["enabled_with_span_ns"] = per_op_ns(guards, a.spans)
    with tempfile.TemporaryDirectory() as d:
        n_spans = len(prof.get_all_spans())
        t0 = time.perf_counter()
        prof.export_chrome_trace(os.path.join(d, "trace.json"))
        out["chrome_trace_export_ms"] = (time.perf_counter() - t0) * 1e3
        t0 = time.perf_counter()
        prof.export_json(os.path.join(d, "stats.json"))
        out["json_stats_export_ms"] = (time.perf_counter() - t0) * 1e3
        out["exported_spans"] = n_spans
    print(json.dumps(out))


if __name__ == "__main__":
    main()
