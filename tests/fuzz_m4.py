"""The reference's differential fuzzer on the B200 (src/gpu/harness-m4.js:125-172, runFuzzM4).

For corpus program i: its forward and gradient runs (naive and tiled when it has a matmul), each the
fused graph and the unfused graph on the GPU judged against the float64 oracle with amendment 8's
budget at every node (runPair, harness-m4.js:78-105), and fused vs unfused compared bit for bit.  A
program with any unjudgeable run is skipped, as the reference does.

    python tests/fuzz_m4.py --out gpurun_out/fuzz.json [--every 1]      # the full corpus: 2000 programs
"""
import argparse
import importlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def program_runs(pkg, co, i):
    """programRunsM4 (harness-m4.js:126-141)."""
    p = co.corpus_program(i, f32=True)
    rng = pkg.rng.Rng((i * 7919 + 17) & 0xFFFFFFFF)
    inputs = {n.attrs["name"]: rng.array(pkg.ir.size(n.shape), -2, 2) for n in p.graph.inputs()}
    G = pkg.autodiff.grad(p.graph, p.outputs, [n.id for n in p.graph.inputs()])
    grad_inputs = dict(inputs)
    for k, name in enumerate(G.cotangents):
        grad_inputs[name] = rng.array(pkg.ir.size(p.graph.nodes[p.outputs[k]].shape), -1, 1)
    has_mm = any(n.op == "matmul" for n in p.graph.nodes)
    runs = []
    for mm in (("naive", "tiled") if has_mm else ("naive",)):
        runs.append({"label": "forward", "graph": p.graph, "inputs": inputs, "outputs": list(p.outputs), "matmul": mm})
        runs.append({"label": "gradient", "graph": G.graph, "inputs": grad_inputs,
                     "outputs": list(p.outputs) + list(G.grads), "matmul": mm})
    return runs


def select(every):
    return [i for i in range(1, 2001) if every == 1 or (i % every) in (1, 2)]


def precompile(pkg, co, programs):
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    codes = set()
    for i in programs:
        for r in program_runs(pkg, co, i):
            f = pkg.fuse.fuse(r["graph"], keep=r["outputs"])
            codes |= {l.code for l in cg.lower_fused(f.graph, matmul=r["matmul"])["launches"]}
            codes |= {l.code for l in cg.lower(r["graph"], matmul=r["matmul"])["launches"]}
    return rt.precompile(codes, threads=min(64, os.cpu_count() or 8))


def run_fuzz(runner, programs, log=None):
    pkg = importlib.import_module("tensor-compiler-webgpu_b200")
    co = importlib.import_module("tensor-compiler-webgpu_b200.corpus")
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    import oracle
    res = {"programs": len(programs), "skipped": 0, "runs": 0, "fusedRuns": 0, "unfusedPassed": 0, "fusedPassed": 0,
           "bitwiseSame": 0, "worstFused": 0.0, "worstUnfused": 0.0, "failures": [], "byKind": {}}
    for i in programs:
        runs = program_runs(pkg, co, i)
        refs = [oracle.reference_with_bounds(r["graph"], r["inputs"]) for r in runs]
        if any(oracle.unjudgeable(v, b) > 0 for v, b, _ in refs):
            res["skipped"] += 1
            continue
        for r, (values, bounds, rounded) in zip(runs, refs):
            res["runs"] += 1
            f = pkg.fuse.fuse(r["graph"], keep=r["outputs"])
            kinds = sorted({n.attrs["kind"] for n in f.graph.nodes if n.op == "fused"})
            if kinds:
                res["fusedRuns"] += 1
            for k in kinds:
                res["byKind"][k] = res["byKind"].get(k, 0) + 1
            gf = runner.run(f.graph, cg.lower_fused(f.graph, matmul=r["matmul"]), rounded)
            jf = oracle.judge_fused(f, gf["values"], values, bounds)
            gu = runner.run(r["graph"], cg.lower(r["graph"], matmul=r["matmul"]), rounded)
            ju = oracle.judge(r["graph"], gu["values"], values, bounds)
            res["fusedPassed"] += jf["pass"]
            res["unfusedPassed"] += ju["pass"]
            res["worstFused"] = max(res["worstFused"], jf["worst"])
            res["worstUnfused"] = max(res["worstUnfused"], ju["worst"])
            same = all(np.array_equal(gf["values"][n.id].view(np.uint32), gu["values"][f.origin[n.id]].view(np.uint32))
                       for n in f.graph.nodes)
            res["bitwiseSame"] += same
            if not (jf["pass"] and ju["pass"]):
                res["failures"].append({"index": i, "run": r["label"], "matmul": r["matmul"], "fused": jf["first"],
                                        "unfused": ju["first"]})
        if log and i % 100 == 0:
            log(f"fuzz {i}: {res['runs']} runs, {len(res['failures'])} failures")
    return res


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--every", type=int, default=1)
    a = ap.parse_args()
    pkg = importlib.import_module("tensor-compiler-webgpu_b200")
    co = importlib.import_module("tensor-compiler-webgpu_b200.corpus")
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    progs = select(a.every)
    print("precompiled", precompile(pkg, co, progs), flush=True)
    runner = rt.GpuRunner.create(0)
    res = run_fuzz(runner, progs, log=lambda m: print(m, flush=True))
    runner.close()
    json.dump(res, open(a.out, "w"), indent=1)
    print(json.dumps({k: v for k, v in res.items() if k != "failures"}), flush=True)
    print("failures", len(res["failures"]), flush=True)
