"""The timing harness (src/fusion/bench.js's protocol) on the B200: a sweep workload's variants
prepared, gated on their outputs against the float64 oracle before anything is timed
(web/m4-bench.html:116-146, src/fusion/workloads.js:351-367), timed in ABBA order with nothing
allocated or compiled inside the timed region (bench.js:201-208), and the ceiling programs moving their
bytes.  A judge that fails a variant keeps the workload from being timed; the model workloads, whose
composed bound is vacuous, are gated on fused versus unfused instead."""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _judge(oracle):
    def judge(graph, inputs, outputs, gpu):
        values, bounds, _ = oracle.reference_with_bounds(graph, inputs, want=list(outputs))
        return oracle.judge_outputs([values[o] for o in outputs], [bounds[o] for o in outputs], gpu)
    return judge


def test_bench_protocol_on_a_sweep_workload(pkg, oracle):
    tm = importlib.import_module("tensor-compiler-webgpu_b200.timing")
    w = next(x for x in tm.workloads() if x["id"] == "softmax-R4096-C256")
    v = tm.build_variants(w)
    bench = tm.Bench.create(0)
    try:
        prepared = {k: bench.prepare(p) for k, p in v["programs"].items()}
        g = tm.gate(bench, w, v, prepared, _judge(oracle))
        assert g["pass"], g
        assert set(g["variants"]) == {"unfused", "fused"} and all(r["elements"] > 0 for r in g["variants"].values())
        for p in prepared.values():
            bench.reset(p)
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


def test_sweep_gates_before_timing(pkg, oracle):
    """run_sweep records each workload's gate; a judge that rejects every variant leaves it untimed."""
    tm = importlib.import_module("tensor-compiler-webgpu_b200.timing")
    bench = tm.Bench.create(0)
    try:
        res = tm.run_sweep(bench, only=["chain-unary-L4-n65537", "forward-V16-B8"], judge=_judge(oracle))
        assert [r["id"] for r in res] == ["chain-unary-L4-n65537", "forward-V16-B8"]
        for r in res:
            assert r["gate"]["pass"], r["gate"]
            assert r["variants"] and all(v["GBps"] > 0 for v in r["variants"].values())
        assert "fusedVsUnfused" in res[1]["gate"]["variants"]

        def reject(graph, inputs, outputs, gpu):
            return {"pass": False, "worst": float("inf")}
        res = tm.run_sweep(bench, only=["chain-unary-L4-n65537"], judge=reject)
        assert res[0]["failedGate"] == ["unfused", "fused"] and res[0]["variants"] == {}
        with pytest.raises(ValueError):
            tm.run_sweep(bench, only=["chain-unary-L4-n65537"])
    finally:
        bench.close()
