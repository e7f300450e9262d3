"""Direct adversarial cases for the fused kernels (restating src/fusion/direct-cases-m4.js:52-132).

Small graphs that fuse into an intended kind, on inputs most likely to break
it: sizes 1..100003, off-tile matmuls, rows C in {1..4097}, softmax at
+-[400, 600], -1e4 masks, constant LayerNorm rows.  Each case is
``{name, kind, pattern, graph, inputs, matmul}``; the graph is the unfused
original.  Same seeds and draw rules as the reference (the drawn values can
differ from it in the last bit where JavaScript's Math.exp/log round
differently from Python's).
"""
from __future__ import annotations

import math

from .ir import Graph, size
from .rng import Rng
from .steps import gelu


def _draw(rng, n, lo, hi):
    out = []
    for _ in range(n):
        if lo < 0 < hi and hi > 1e3:
            m = math.exp(rng.uniform(math.log(hi) - 20, math.log(hi)))
            out.append(m if rng.chance(0.5) else -m)
        elif lo > 0 and hi / lo > 100:
            out.append(math.exp(rng.uniform(math.log(lo), math.log(hi))))
        else:
            out.append(rng.uniform(lo, hi))
    return out


def layer_norm_graph(g, x, gain, bias, eps=1e-5):
    """Milestone 3b's LayerNorm over the last axis (direct-cases-m4.js:20-28)."""
    d = g.shape(x)[-1]
    axis = len(g.shape(x)) - 1
    mean = g.div(g.sum(x, axis, True), g.const(d))
    xc = g.sub(x, mean)
    variance = g.div(g.sum(g.mul(xc, xc), axis, True), g.const(d))
    y = g.div(xc, g.sqrt(g.add(variance, g.const(eps))))
    return g.add(g.mul(y, gain), bias)


def unary_chain(g, x, L):
    """tanh, exp, neg, exp, sqrt, log, repeating: values stay finite and in range (direct-cases-m4.js:38-44)."""
    cycle = [g.tanh, g.exp, g.neg, g.exp, g.sqrt, g.log]
    y = x
    for k in range(L):
        y = cycle[k % len(cycle)](y)
    return y


def _one(name, kind, pattern, build, inputs, **extra):
    g = Graph()
    build(g)
    return {"name": name, "kind": kind, "pattern": pattern, "graph": g, "inputs": inputs, **extra}


def fused_direct_cases():
    rng = Rng(20261019)
    cases = []
    SIZES = [[1], [63], [64], [65], [1000], [100003], [3, 5, 7], [1, 7, 1]]
    for shape in SIZES:
        n = size(shape)
        cases.append(_one(f"chain of 6 [{','.join(map(str, shape))}]", "elementwise", "elementwise",
                          lambda g, shape=shape: unary_chain(g, g.input("x", shape), 6), {"x": _draw(rng, n, -2, 2)}))
        ins = {k: _draw(rng, n, -2, 2) for k in "abcd"}
        ins["e"] = _draw(rng, n, 0.5, 2)
        cases.append(_one(f"a*b+c-d/e [{','.join(map(str, shape))}]", "elementwise", "elementwise",
                          lambda g, shape=shape: g.sub(g.add(g.mul(g.input("a", shape), g.input("b", shape)),
                                                             g.input("c", shape)),
                                                       g.div(g.input("d", shape), g.input("e", shape))), ins))
    for cls, (lo, hi) in (("large", (-1e18, 1e18)), ("small", (-1e-18, 1e-18)), ("subnormal", (-1e-40, 1e-40))):
        ins = {"a": _draw(rng, 1000, lo, hi), "b": _draw(rng, 1000, -2, 2), "c": _draw(rng, 1000, lo, hi)}
        cases.append(_one(f"a*b+c {cls} [1000]", "elementwise", "elementwise",
                          lambda g: g.add(g.mul(g.input("a", [1000]), g.input("b", [1000])), g.input("c", [1000])),
                          ins))
    cases.append(_one("relu(x)*2 exact zeros [65]", "elementwise", "elementwise",
                      lambda g: g.mul(g.relu(g.input("x", [65])), g.const(2)), {"x": [0.0] * 65}))
    cases.append(_one("x + broadcast(b) [3,65] <- [65]", "elementwise", "elementwise",
                      lambda g: g.tanh(g.add(g.input("x", [3, 65]), g.input("b", [65]))),
                      {"x": _draw(rng, 195, -2, 2), "b": _draw(rng, 65, -2, 2)}))
    cases.append(_one("x + broadcast(b) [2,4,3,5] <- [2,1,3,1]", "elementwise", "elementwise",
                      lambda g: g.exp(g.sub(g.input("x", [2, 4, 3, 5]), g.input("b", [2, 1, 3, 1]))),
                      {"x": _draw(rng, 120, -2, 2), "b": _draw(rng, 6, -2, 2)}))
    cases.append(_one("transpose(x) * y [5,7] <- [7,5]", "elementwise", "elementwise",
                      lambda g: g.mul(g.transpose(g.input("x", [7, 5]), [1, 0]), g.neg(g.input("y", [5, 7]))),
                      {"x": _draw(rng, 35, -2, 2), "y": _draw(rng, 35, -2, 2)}))
    cases.append(_one("transpose(x) + y [2,3,4] perm [2,0,1]", "elementwise", "elementwise",
                      lambda g: g.add(g.transpose(g.input("x", [3, 4, 2]), [2, 0, 1]), g.exp(g.input("y", [2, 3, 4]))),
                      {"x": _draw(rng, 24, -2, 2), "y": _draw(rng, 24, -2, 2)}))

    MM = [([1, 1], [1, 1]), ([17, 33], [33, 19]), ([15, 16], [16, 17]), ([16, 16], [16, 16]), ([1, 64], [64, 1]),
          ([64, 1], [1, 64]), ([3, 5, 7], [3, 7, 2]), ([2, 17, 19], [2, 19, 33]), ([3, 4096], [4096, 5])]
    for matmul in ("naive", "tiled"):
        for a_s, b_s in MM:
            N = b_s[-1]
            for act in ("relu", "gelu"):
                def build(g, a_s=a_s, b_s=b_s, N=N, act=act):
                    y = g.add(g.matmul(g.input("a", a_s), g.input("w", b_s)), g.input("bias", [N]))
                    return g.relu(y) if act == "relu" else gelu(g, y)
                ins = {"a": _draw(rng, size(a_s), -2, 2), "w": _draw(rng, size(b_s), -2, 2), "bias": _draw(rng, N, -2, 2)}
                cases.append(_one(f"matmul {matmul} [{','.join(map(str, a_s))}] x [{','.join(map(str, b_s))}] + bias, {act}",
                                  "epilogue", "matmul-epilogue", build, ins, matmul=matmul))
        ins = {"a": _draw(rng, 561, -1e15, 1e15), "w": _draw(rng, 627, -1e15, 1e15), "bias": _draw(rng, 19, -1e30, 1e30)}
        cases.append(_one(f"matmul {matmul} [17,33] x [33,19] + bias, relu, large", "epilogue", "matmul-epilogue",
                          lambda g: g.relu(g.add(g.matmul(g.input("a", [17, 33]), g.input("w", [33, 19])),
                                                 g.input("bias", [19]))), ins, matmul=matmul))
        ins = {"a": _draw(rng, 561, -2, 2), "w": _draw(rng, 627, -2, 2), "bias": _draw(rng, 19, -2, 2),
               "res": _draw(rng, 323, -2, 2)}
        cases.append(_one(f"matmul {matmul} [17,33] x [33,19] + residual", "epilogue", "matmul-epilogue",
                          lambda g: g.add(g.add(g.matmul(g.input("a", [17, 33]), g.input("w", [33, 19])),
                                                g.input("bias", [19])), g.input("res", [17, 19])), ins, matmul=matmul))

    ROWS = [(1, 1), (3, 7), (65, 63), (2, 64), (3, 65), (2, 257), (3, 1000), (1, 4097)]
    for R, C in ROWS:
        if C > 1:
            ins = {"x": _draw(rng, R * C, -2, 2)}
            ins.update({"g": _draw(rng, C, 0.5, 2), "b": _draw(rng, C, -1, 1)})
            cases.append(_one(f"layernorm [{R},{C}]", "rowwise", "layernorm",
                              lambda g, R=R, C=C: layer_norm_graph(g, g.input("x", [R, C]), g.input("g", [C]),
                                                                   g.input("b", [C])), ins))
            cases.append(_one(f"softmax [{R},{C}]", "rowwise", "softmax",
                              lambda g, R=R, C=C: g.softmax(g.input("x", [R, C]), 1), {"x": _draw(rng, R * C, -2, 2)}))
            cases.append(_one(f"log-softmax [{R},{C}]", "rowwise", "log-softmax",
                              lambda g, R=R, C=C: g.log_softmax(g.input("x", [R, C]), 1),
                              {"x": _draw(rng, R * C, -2, 2)}))
    cases.append(_one("layernorm [4,64] constant rows", "rowwise", "layernorm",
                      lambda g: layer_norm_graph(g, g.input("x", [4, 64]), g.input("g", [64]), g.input("b", [64])),
                      {"x": [[0, 1, -3, 10][i >> 6] for i in range(256)], "g": _draw(rng, 64, 0.5, 2),
                       "b": _draw(rng, 64, -1, 1)}))
    cases.append(_one("layernorm [3,65] far from zero", "rowwise", "layernorm",
                      lambda g: layer_norm_graph(g, g.input("x", [3, 65]), g.input("g", [65]), g.input("b", [65])),
                      {"x": _draw(rng, 195, 1000, 1001), "g": _draw(rng, 65, 0.5, 2), "b": _draw(rng, 65, -1, 1)}))
    cases.append(_one("layernorm [2,3,64] rank 3", "rowwise", "layernorm",
                      lambda g: layer_norm_graph(g, g.input("x", [2, 3, 64]), g.input("g", [64]), g.input("b", [64])),
                      {"x": _draw(rng, 384, -2, 2), "g": _draw(rng, 64, 0.5, 2), "b": _draw(rng, 64, -1, 1)}))
    for op in ("softmax", "logSoftmax"):
        pattern = "softmax" if op == "softmax" else "log-softmax"
        fn = "softmax" if op == "softmax" else "log_softmax"

        def sm(shape, fn=fn):
            return lambda g: getattr(g, fn)(g.input("x", shape), len(shape) - 1)
        for label, (lo, hi) in (("large", (400, 600)), ("large negative", (-600, -400)), ("small", (-1e-30, 1e-30))):
            cases.append(_one(f"{pattern} {label} [3,65]", "rowwise", pattern, sm([3, 65]), {"x": _draw(rng, 195, lo, hi)}))
        cases.append(_one(f"{pattern} exact zeros [3,65]", "rowwise", pattern, sm([3, 65]), {"x": [0.0] * 195}))
        mask = [0 if j <= i else -1e4 for i in range(64) for j in range(64)]
        cases.append(_one(f"{pattern} masked [2,64,64]", "rowwise", pattern,
                          lambda g, fn=fn, mask=mask: getattr(g, fn)(g.add(g.input("x", [2, 64, 64]),
                                                                           g.const(mask, [64, 64])), 2),
                          {"x": _draw(rng, 8192, -13, 13)}))
        cases.append(_one(f"{pattern} [2,4,8,65] rank 4", "rowwise", pattern, sm([2, 4, 8, 65]),
                          {"x": _draw(rng, 4160, -2, 2)}))
    return cases
