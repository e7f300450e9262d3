"""The timing harness (src/fusion/bench.js's protocol) on the B200: a sweep workload's variants
prepared, their outputs agreeing, timed in ABBA order with nothing allocated or compiled inside the
timed region (bench.js:201-208), and the ceiling programs moving their bytes."""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bench_protocol_on_a_sweep_workload(pkg):
    tm = importlib.import_module("tensor-compiler-webgpu_b200.timing")
    w = next(x for x in tm.workloads() if x["id"] == "softmax-R4096-C256")
    v = tm.build_variants(w)
    bench = tm.Bench.create(0)
    try:
        prepared = {k: bench.prepare(p) for k, p in v["programs"].items()}
        outs = {k: bench.outputs(p) for k, p in prepared.items()}
        for a, b in zip(outs["unfused"], outs["fused"]):
            np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-7)
        t = bench.time(prepared)
        assert t["created"] == {}
        assert t["k"] >= 1 and all(len(r) == tm.REPS for r in t["reps"].values())
        s = {k: tm.summarize(r) for k, r in t["reps"].items()}
        assert s["fused"]["gpuNs"]["median"] < s["unfused"]["gpuNs"]["median"]  # fewer launches, fewer bytes
        for p in prepared.values():
            bench.destroy(p)
        c = next(x for x in tm.ceiling_programs() if x["id"] == "copy-vec4-x4096")
        p = bench.prepare(c["program"])
        t = bench.time({"c": p})
        gbps = c["program"]["bytes"] / tm.summarize(t["reps"]["c"])["gpuNs"]["median"]
        assert gbps > 2000, gbps
        bench.destroy(p)
    finally:
        bench.close()
