"""The reference's golden cases through the CUDA path: fused and unfused, every node within 2E.

golden/cases.json (112 cases: softmax and logSoftmax with "large" 800-range rows, mlp-nll, attention,
transpose cycles, random graphs) and golden/cases-m3.json (34 sqrt cases), each as the forward graph
plus its autodiff backward with the recorded cotangents.  The PyTorch float64 goldens pin the oracle
(tests/test_oracle_golden.py); here the oracle's values and amendment 8 bounds judge the B200, by the
protocol of src/gpu/harness-m4.js:78-121: the fused graph with canary-padded buffers and every
surviving node judged, then the unfused graph judged node by node.  A reference outside float32's range
or with an unbounded error makes a case unjudgeable (harness-m4.js:80): such cases are counted, and at
most a few may be.  Both matmul paths run: the CUDA-core kernel ('naive') and the tcgen05 3xTF32 kernel
('tiled', used where K >= 32).
"""
import importlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _cases():
    with open(os.path.join(GOLDEN, "cases_torch.json")) as f:
        a = json.load(f)["cases"]
    with open(os.path.join(GOLDEN, "cases_m3_torch.json")) as f:
        b = json.load(f)["cases"]["cases"]
    return a + b


CASES = _cases()


def _graph_of(pkg, c):
    g = pkg.ir.Graph.from_json(c["graph"])
    inputs = g.inputs()
    G = pkg.autodiff.grad(g, c["outputs"], [n.id for n in inputs])
    feed = dict(c["inputs"])
    for i, name in enumerate(G.cotangents):
        feed[name] = c["cotangents"][i]
    return G.graph, feed, list(c["outputs"]) + list(G.grads)


@pytest.mark.parametrize("matmul", ["naive", "tiled"])
def test_golden_cases_on_the_gpu(pkg, oracle, runner, matmul):
    assert len(CASES) == 146
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    skipped, failed, judged = [], [], 0
    for c in CASES:
        graph, feed, keep = _graph_of(pkg, c)
        values, bounds, rounded = oracle.reference_with_bounds(graph, feed)
        if oracle.unjudgeable(values, bounds) > 0:
            skipped.append(c["name"])
            continue
        fused = pkg.fuse.fuse(graph, keep=keep)
        gf = runner.run(fused.graph, cg.lower_fused(fused.graph, matmul=matmul), rounded, canary=True)
        jf = oracle.judge_fused(fused, gf["values"], values, bounds)
        gu = runner.run(graph, cg.lower(graph, matmul=matmul), rounded, canary=True)
        ju = oracle.judge(graph, gu["values"], values, bounds)
        ok = jf["pass"] and ju["pass"] and all(gf["canaryIntact"]) and all(gu["canaryIntact"])
        if not ok:
            failed.append((c["name"], jf["first"], ju["first"]))
        judged += 1
    assert not failed, failed[:5]
    assert len(skipped) <= 4, skipped
    assert judged + len(skipped) == len(CASES)
