"""The reference's value sabotages run on the B200: the 2E judge must catch each planted kernel bug.

src/gpu/harness-m4.js:364-403 (runSabotageM4, direct phase): every direct case is run honestly and then
with one bug planted in the generated fused kernels (FUSED_SABOTAGE, src/fusion/codegen-fused.js:22);
a case is caught when it passed honestly and its sabotaged fused values fail the judge.  The three bugs
here compute wrong numbers but stay inside their buffers and end normally:

* epilogue-before-bias: the fused matmul epilogue applies its activation before adding the bias;
* layernorm-tree-short: the rowwise reduction skips its cross-thread combine step;
* softmax-no-max: softmax / logSoftmax take no max shift (rows near +800 overflow).

The fourth, fused-bounds-off-by-one, writes one element past the output and is checked on the CPU
only (tests/test_sabotage_cpu.py).  The reference's own record (golden/gpu-m4.json) caught 31, 10 and 4
of its 100 cases; the caught cases must all be ones the bug can reach (its kind or pattern).
"""
import importlib

import pytest

pytestmark = pytest.mark.gpu

TARGET = {"epilogue-before-bias": ("kind", {"epilogue"}),
          "layernorm-tree-short": ("pattern", {"layernorm"}),
          "softmax-no-max": ("pattern", {"softmax", "log-softmax"})}


def _run(pkg, oracle, runner, case, sabotage=None):
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    graph = case["graph"]
    values, bounds, rounded = oracle.reference_with_bounds(graph, case["inputs"])
    if oracle.unjudgeable(values, bounds) > 0:
        return None, None
    fused = pkg.fuse.fuse(graph)
    lowered = cg.lower_fused(fused.graph, matmul=case.get("matmul", "naive"), sabotage=sabotage)
    gf = runner.run(fused.graph, lowered, rounded, canary=True)
    j = oracle.judge_fused(fused, gf["values"], values, bounds)
    return j["pass"] and all(gf["canaryIntact"]), fused


@pytest.mark.parametrize("sabotage", sorted(TARGET))
def test_value_sabotage_is_caught_on_the_gpu(pkg, oracle, runner, sabotage):
    cases = importlib.import_module("tensor-compiler-webgpu_b200.cases").fused_direct_cases()
    assert len(cases) == 100
    field, targets = TARGET[sabotage]
    caught, honest_pass, reachable = [], 0, 0
    for case in cases:
        ok, fused = _run(pkg, oracle, runner, case)
        if ok is None or not ok:
            continue
        honest_pass += 1
        nodes = [n for n in fused.graph.nodes if n.op == "fused"]
        reach = any(n.attrs[field] in targets for n in nodes)
        reachable += reach
        bad, _ = _run(pkg, oracle, runner, case, sabotage)
        if bad is False:
            caught.append(case["name"])
            assert reach, f"{case['name']}: caught, but {sabotage} cannot reach it"
    assert honest_pass >= 95
    assert caught, f"{sabotage}: no case caught ({reachable} reachable)"
    print(f"{sabotage}: caught {len(caught)} of {honest_pass} honest passes ({reachable} reachable): {caught}")
