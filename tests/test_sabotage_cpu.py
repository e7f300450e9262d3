"""The judges catch planted mistakes: each of the reference's kernel sabotages
(src/fusion/codegen-fused.js:22, harness-m4.js:34-40) planted in the oracle on the CPU.

Running kernels broken on purpose on the shared GPUs is closed on this pool, so the mistake is
planted in the float64 evaluation instead and the same budget judge must flag it.
"""
import importlib

import numpy as np
import pytest


def _case(name):
    cases = importlib.import_module("tensor-compiler-webgpu_b200.cases").fused_direct_cases()
    return next(c for c in cases if c["name"] == name)


def _judged(oracle, graph, inputs, bad_graph):
    values, bounds, rounded = oracle.reference_with_bounds(graph, inputs)
    bad = oracle.evaluate(bad_graph, rounded)
    f32 = [None if v is None else np.asarray(v, dtype=np.float32) for v in bad]
    return oracle.judge(graph, f32, values, bounds)


def test_softmax_without_max_is_caught(pkg, oracle):
    c = _case("softmax large [3,65]")
    g = c["graph"]
    bad = g.clone()
    for n in bad.nodes:  # the shift is never taken: stopGradient(max) becomes 0
        if n.op == "stopGradient":
            n.op, n.inputs, n.attrs = "const", [], {"shape": list(n.shape), "value": 0}
    j = _judged(oracle, g, c["inputs"], bad)
    assert not j["pass"]


def test_epilogue_before_bias_is_caught(pkg, oracle):
    c = _case("matmul naive [17,33] x [33,19] + bias, relu")
    g = c["graph"]
    # relu(matmul) + bias instead of relu(matmul + bias)
    bad = pkg.ir.Graph()
    a = bad.input("a", [17, 33]); w = bad.input("w", [33, 19]); b = bad.input("bias", [19])
    bad.add(bad.relu(bad.matmul(a, w)), b)
    values, bounds, rounded = oracle.reference_with_bounds(g, c["inputs"])
    wrong = oracle.evaluate(bad, rounded)
    out = [n.id for n in g.nodes][-1]
    r = oracle._ratio(np.asarray(wrong[-1], np.float32), values[out], bounds[out])
    assert float(r.max()) > 1


def test_layernorm_short_tree_is_caught(pkg, oracle):
    c = _case("layernorm [3,65]")
    g = c["graph"]
    values, bounds, rounded = oracle.reference_with_bounds(g, c["inputs"])
    # the tree stops one level early: each row's sums miss the second half of the row
    x = rounded["x"].reshape(3, 65)
    short = x.copy()
    short[:, 33:] = 0
    wrong = oracle.evaluate(g, {**rounded, "x": short.reshape(-1)})
    out = len(g.nodes) - 1
    r = oracle._ratio(np.asarray(wrong[out], np.float32), values[out], bounds[out])
    assert float(r.max()) > 1


def test_fusion_absorbing_a_shared_value_is_caught(pkg, oracle):
    # a shared producer consumed outside the group: the sabotaged pass changes semantics or throws
    g = pkg.ir.Graph()
    x = g.input("x", [8])
    t = g.exp(x)
    u = g.tanh(t)
    v = g.add(u, t)
    w = g.mul(t, g.const(3))
    inputs = {"x": np.linspace(-1, 1, 8)}
    honest = pkg.fuse.fuse(g, keep=[v, w])
    assert oracle.check_semantics(g, honest, inputs)["identical"]
    try:
        bad = pkg.fuse.fuse(g, keep=[v, w], sabotage="fusion-absorbs-shared")
    except RuntimeError:
        return
    assert not oracle.check_semantics(g, bad, inputs)["identical"]
