"""The BASELINE workloads (C1-C5) as graphs plus seeded synthetic inputs.

Every input comes from mulberry32 (src/testing/rng.js) seeded 0 unless
stated; normal draws are Box-Muller over it (rng.normal_array).  The shapes,
value distributions and graph forms follow BASELINE.json's configs; the
reference has no such workloads of its own (its sweep is
src/fusion/workloads.js:76-126), so each builder states its choices.

C2's chain: 8 ops drawn with ``Rng(0).pick`` from {add, mul, sub, div, exp,
log, tanh, relu, neg}.  The running value starts at x0 [R, C] ~ N(0,1).  A
binary op combines it with a fresh [R, C] input -- except the first binary
op, whose operand is the [1, C] row ``r`` broadcast over rows; add/sub/mul
operands ~ N(0,1), div denominators ~ U[0.5, 2].  Unary ops apply to the
running value.  So that every value stays finite and inside log's domain, a
drawn ``exp`` directly after ``exp`` and a drawn ``log`` not directly after
``exp`` are redrawn from the same stream.  Forward + backward: the gradient
of the chain output with respect to every input, cotangent d0 ~ N(0,1).
"""
from __future__ import annotations

import numpy as np

from .autodiff import grad
from .ir import Graph, size
from .rng import Rng
from . import steps as _steps

C2_OPS = ("add", "mul", "sub", "div", "exp", "log", "tanh", "relu", "neg")
BINARY = ("add", "mul", "sub", "div")


def c2_ops(seed=0, length=8):
    rng = Rng(seed)
    ops = []
    while len(ops) < length:
        op = rng.pick(C2_OPS)
        prev = ops[-1] if ops else None
        if op == "exp" and prev == "exp":
            continue
        if op == "log" and prev != "exp":
            continue
        ops.append(op)
    return ops


def c2_graph(R=8192, C=8192, seed=0):
    """The C2 chain: forward + autodiff backward.  Returns a dict like the step builders'."""
    ops = c2_ops(seed)
    g = Graph()
    x0 = g.input("x0", [R, C])
    dist = {"x0": ("normal",)}
    v = x0
    first_binary = True
    k = 0
    for op in ops:
        if op in BINARY:
            if first_binary:
                name, shape = "r", [1, C]
                first_binary = False
            else:
                k += 1
                name, shape = f"x{k}", [R, C]
            dist[name] = ("uniform", 0.5, 2.0) if op == "div" else ("normal",)
            operand = g.input(name, shape)
            v = getattr(g, op)(v, operand)
        else:
            v = getattr(g, op)(v)
    wrt = [n.id for n in g.inputs()]
    G = grad(g, [v], wrt)
    names = [g.nodes[i].attrs["name"] for i in wrt]
    return {"graph": G.graph, "forward": g, "ops": ops, "output": v, "grads": dict(zip(names, G.grads)),
            "cotangent": G.cotangents[0], "dist": dist, "keep": [v, *G.grads], "R": R, "C": C}


def c2_inputs(w, seed=0):
    """Seeded float32 inputs for a c2_graph: each input drawn in graph order from one stream."""
    rng = Rng(seed)
    out = {}
    g = w["graph"]
    for node in g.inputs():
        name = node.attrs["name"]
        n = size(node.shape)
        d = w["dist"].get(name, ("normal",))
        if d[0] == "uniform":
            out[name] = rng.uniform_array(n, d[1], d[2]).astype(np.float32)
        else:
            out[name] = rng.normal_array(n).astype(np.float32)
    return out


# ---------------------------------------------------------------- C1: MLP 64 -> 32 -> 10
C1_DIMS = {"inputs": 64, "hidden": 32, "classes": 10}


def c1_step(batch=64, opt=None):
    """matmul + bias + tanh -> matmul + bias -> logSoftmax -> mean NLL, with gradients (opt None: no update)."""
    return _steps.build_mlp_step(C1_DIMS, batch, opt=opt, hidden="tanh")


def c1_inputs(batch=64, seed=0):
    """Features int(0..16)/16, labels uniform 0..9 one-hot, Glorot-normal weights, zero biases."""
    rng = Rng(seed)
    d = C1_DIMS
    x = np.array([rng.int(0, 16) / 16 for _ in range(batch * d["inputs"])], dtype=np.float32)
    labels = [rng.int(0, d["classes"] - 1) for _ in range(batch)]
    y = np.zeros((batch, d["classes"]), dtype=np.float32)
    y[np.arange(batch), labels] = 1
    s1 = np.sqrt(2 / (d["inputs"] + d["hidden"]))
    s2 = np.sqrt(2 / (d["hidden"] + d["classes"]))
    params = {"W1": rng.normal_array(d["inputs"] * d["hidden"], 0, s1).astype(np.float32),
              "b1": np.zeros(d["hidden"], np.float32),
              "W2": rng.normal_array(d["hidden"] * d["classes"], 0, s2).astype(np.float32),
              "b2": np.zeros(d["classes"], np.float32)}
    return {**params, "x": x, "y": y.reshape(-1)}


# ---------------------------------------------------------------- C3: matmul + bias + activation
C3_SHAPES = ((4096, 4096, 4096), (16384, 1024, 4096))


def c3_graph(M, K, N, act="relu"):
    g = Graph()
    a = g.input("a", [M, K])
    b = g.input("b", [K, N])
    bias = g.input("bias", [N])
    y = g.add(g.matmul(a, b), bias)
    out = g.relu(y) if act == "relu" else g.tanh(y)
    return {"graph": g, "output": out, "keep": [out], "M": M, "K": K, "N": N, "act": act}


def c3_inputs(M, K, N, seed=0, rows=None):
    """A, B ~ N(0, 1/K) (std 1/sqrt(K)), bias ~ N(0, 0.1) (std sqrt(0.1))."""
    rng = Rng(seed)
    s = 1 / np.sqrt(K)
    a = rng.normal_array(M * K, 0, s).astype(np.float32)
    b = rng.normal_array(K * N, 0, s).astype(np.float32)
    bias = rng.normal_array(N, 0, np.sqrt(0.1)).astype(np.float32)
    return {"a": a, "b": b, "bias": bias}


# ---------------------------------------------------------------- C4: rowwise softmax / logSoftmax / row sum
def c4_graph(R=65536, C=4096, what="softmax"):
    """Forward and backward of softmax, logSoftmax or a row sum over the last axis."""
    g = Graph()
    x = g.input("x", [R, C])
    if what == "softmax":
        y = g.softmax(x, 1)
    elif what == "logsoftmax":
        y = g.log_softmax(x, 1)
    else:
        y = g.sum(x, 1, True)
    G = grad(g, [y], [x])
    return {"graph": G.graph, "forward": g, "output": y, "grad": G.grads[0], "cotangent": G.cotangents[0],
            "keep": [y, G.grads[0]], "R": R, "C": C, "what": what}


def c4_inputs(w, seed=0):
    """Logits ~ N(0, 4) (std 2); 1% of rows (seeded) offset by +800; upstream gradient ~ N(0, 1)."""
    R, C = w["R"], w["C"]
    rng = Rng(seed)
    x = rng.normal_array(R * C, 0, 2.0).reshape(R, C)
    hot = max(1, R // 100)
    rows = sorted(set(int(v) for v in np.floor(rng.next_array(4 * hot) * R)))[:hot]
    x[rows] += 800.0
    out_shape = w["forward"].nodes[w["output"]].shape
    d0 = rng.normal_array(size(out_shape)).astype(np.float32)
    return {"x": x.astype(np.float32).reshape(-1), w["cotangent"]: d0}, rows


# ---------------------------------------------------------------- C5: decoder transformer
C5_CONFIG = {"V": 65, "d": 256, "L": 4, "H": 4, "ff": 1024, "T": 256, "batch": 512}


def c5_cfg(**over):
    c = dict(C5_CONFIG)
    c.update(over)
    return _steps.make_config(T=c["T"], d=c["d"], H=c["H"], L=c["L"], ff=c["ff"]), c


def c5_tokens(batch, T, V, seed=0):
    """Token sequences of T+1 tokens uniform over 0..V-1 (mulberry32)."""
    rng = Rng(seed)
    toks = np.floor(rng.next_array(batch * (T + 1)) * V).astype(np.int64).reshape(batch, T + 1)
    return toks


def one_hot_batch(toks, V):
    B, T1 = toks.shape
    T = T1 - 1
    x = np.zeros((B * T, V), dtype=np.float32)
    y = np.zeros((B * T, V), dtype=np.float32)
    rows = np.arange(B * T)
    x[rows, toks[:, :T].reshape(-1)] = 1
    y[rows, toks[:, 1:].reshape(-1)] = 1
    return x.reshape(-1), y.reshape(-1)
