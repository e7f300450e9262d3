"""The fused kernels on the B200 against the float64 oracle: the reference's 100 direct cases.

Protocol of src/gpu/harness-m4.js:78-121 (runPair, runDirectM4): the graph's
reference with amendment 8's bounds (inputs rounded to float32 first), the
fused graph run with canary-padded buffers, every surviving node judged at
|gpu - ref| <= 2E, every canary intact; the unfused graph judged the same way
and compared with the fused one bit for bit (a rate that is reported, not
required).
"""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _cases():
    return importlib.import_module("tensor-compiler-webgpu_b200.cases").fused_direct_cases()


CASES = _cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_direct_case(pkg, oracle, runner, case):
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    graph = case["graph"]
    values, bounds, rounded = oracle.reference_with_bounds(graph, case["inputs"])
    if oracle.unjudgeable(values, bounds) > 0:
        pytest.skip("reference not judgeable (harness-m4.js:80)")
    fused = pkg.fuse.fuse(graph)
    kinds = {n.attrs["kind"] for n in fused.graph.nodes if n.op == "fused"}
    assert kinds == {case["kind"]}
    matmul = case.get("matmul", "naive")
    gf = runner.run(fused.graph, cg.lower_fused(fused.graph, matmul=matmul), rounded, canary=True)
    j = oracle.judge_fused(fused, gf["values"], values, bounds)
    assert all(gf["canaryIntact"]), "a fused kernel wrote past its output"
    assert j["pass"], j["first"]
    gu = runner.run(graph, cg.lower(graph, matmul=matmul), rounded, canary=True)
    ju = oracle.judge(graph, gu["values"], values, bounds)
    assert all(gu["canaryIntact"]), "an unfused kernel wrote past its output"
    assert ju["pass"], ju["first"]
    same = all(np.array_equal(gf["values"][n.id].view(np.uint32), gu["values"][fused.origin[n.id]].view(np.uint32))
               for n in fused.graph.nodes)
    case["bitwise_same"] = same
