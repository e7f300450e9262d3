"""Graph sources: the MLP step, the decoder transformer and Adam, built from IR ops.

Restates the reference's step builders so the backend has its graphs:
``src/train/step.js:49-116`` (MLP step; ``hidden`` activation selectable so
the tanh MLP of the C1 workload can be built), ``src/m3b/model.js:29-145``
(pre-LN decoder), ``src/m3b/adam.js:8-48`` (Adam from ops) and
``src/m3b/step.js:13-31`` (forward + grad + Adam).  The reference hard-codes
the transformer's sizes (src/m3b/model.js:12); here they are a ``cfg`` dict
whose default is that same CONFIG.
"""
from __future__ import annotations

import math

from .autodiff import grad
from .ir import Graph
from .rng import Rng

# ---------------------------------------------------------------- MLP (src/train/step.js)
PARAMS = ("W1", "b1", "W2", "b2")
SGD = {"kind": "sgd", "lr": 0.1, "momentum": 0.9, "weightDecay": 5e-4}
ADAM = {"kind": "adam", "lr": 0.01, "beta1": 0.9, "beta2": 0.999, "eps": 1e-8, "weightDecay": 1e-4}


def _mlp_shapes(dims):
    return {"W1": [dims["inputs"], dims["hidden"]], "b1": [dims["hidden"]],
            "W2": [dims["hidden"], dims["classes"]], "b2": [dims["classes"]]}


def mlp_state_spec(opt, dims):
    s = _mlp_shapes(dims)
    if opt["kind"] == "sgd":
        return {f"{p}.buf": s[p] for p in PARAMS}
    out = {}
    for p in PARAMS:
        out[f"{p}.m"] = s[p]
        out[f"{p}.v"] = s[p]
    out["beta1Pow"] = []
    out["beta2Pow"] = []
    return out


def mlp_initial_state(opt, dims):
    out = {}
    for name, shape in mlp_state_spec(opt, dims).items():
        n = 1
        for d in shape:
            n *= d
        out[name] = [1.0 if name.endswith("Pow") else 0.0] * n
    return out


def mlp_logits(g, ids, hidden="relu"):
    """x -> act(x W1 + b1) W2 + b2 (src/train/step.js:49-52; act relu there)."""
    pre = g.add(g.matmul(ids["x"], ids["W1"]), ids["b1"])
    h = g.relu(pre) if hidden == "relu" else g.tanh(pre)
    return g.add(g.matmul(h, ids["W2"]), ids["b2"])


def build_mlp_step(dims, batch, opt=None, hidden="relu", sabotage=None):
    """The MLP training step graph (src/train/step.js:60-116).

    ``opt=None`` builds forward + mean NLL + gradients only (no update): the
    outputs are then the gradients by parameter name.
    """
    g = Graph()
    s = _mlp_shapes(dims)
    ids = {p: g.input(p, s[p]) for p in PARAMS}
    ids["x"] = g.input("x", [batch, dims["inputs"]])
    ids["y"] = g.input("y", [batch, dims["classes"]])
    logp = g.log_softmax(mlp_logits(g, ids, hidden), 1)
    loss = g.div(g.neg(g.sum(g.sum(g.mul(ids["y"], logp), 1), 0)), g.const(batch))
    G = grad(g, [loss], [ids[p] for p in PARAMS])
    B = G.graph
    grads = {p: G.grads[k] for k, p in enumerate(PARAMS)}
    inputs = {**{p: ids[p] for p in PARAMS}, "x": ids["x"], "y": ids["y"]}
    if opt is None:
        return {"graph": B, "inputs": inputs, "loss": loss, "logits": logp, "outputs": dict(grads),
                "cotangent": G.cotangents[0], "grads": grads}
    state = {name: B.input(name, shape) for name, shape in mlp_state_spec(opt, dims).items()}
    c = B.const
    outputs = {}

    def decayed(p):
        if sabotage == "weight-decay-sign":
            return B.sub(grads[p], B.mul(c(opt["weightDecay"]), ids[p]))
        return B.add(grads[p], B.mul(c(opt["weightDecay"]), ids[p]))

    if opt["kind"] == "sgd":
        for p in PARAMS:
            buf = state[f"{p}.buf"]
            nxt = B.add(B.mul(c(opt["momentum"]), buf), decayed(p))
            used = buf if sabotage == "momentum-off-by-one" else nxt
            outputs[p] = B.sub(ids[p], B.mul(c(opt["lr"]), used))
            outputs[f"{p}.buf"] = nxt
    else:
        b1 = B.mul(state["beta1Pow"], c(opt["beta1"]))
        b2 = B.mul(state["beta2Pow"], c(opt["beta2"]))
        outputs["beta1Pow"] = b1
        outputs["beta2Pow"] = b2
        bc1 = B.sub(c(1), b1)
        bc2 = B.sub(c(1), b1 if sabotage == "adam-bias-correction" else b2)
        step_size = B.div(c(opt["lr"]), bc1)
        sqrt_bc2 = B.sqrt(bc2)
        for p in PARAMS:
            gp = decayed(p)
            m = B.add(B.mul(c(opt["beta1"]), state[f"{p}.m"]), B.mul(c(1 - opt["beta1"]), gp))
            v = B.add(B.mul(c(opt["beta2"]), state[f"{p}.v"]), B.mul(c(1 - opt["beta2"]), B.mul(gp, gp)))
            denom = B.add(B.div(B.sqrt(v), sqrt_bc2), c(opt["eps"]))
            outputs[p] = B.sub(ids[p], B.mul(step_size, B.div(m, denom)))
            outputs[f"{p}.m"] = m
            outputs[f"{p}.v"] = v
    inputs.update(state)
    return {"graph": B, "inputs": inputs, "loss": loss, "logits": logp, "outputs": outputs,
            "cotangent": G.cotangents[0], "grads": grads}


# ---------------------------------------------------------------- transformer (src/m3b/model.js)
CONFIG = {"T": 64, "d": 64, "H": 4, "dh": 16, "L": 2, "ff": 256, "eps": 1e-5, "mask": -1e4}


def make_config(**kw):
    cfg = dict(CONFIG)
    cfg.update(kw)
    cfg["dh"] = cfg["d"] // cfg["H"]
    return cfg


def param_spec(V, cfg=CONFIG):
    """Parameters in their fixed order: (name, shape, init) (src/m3b/model.js:29-45)."""
    T, d, L, ff = cfg["T"], cfg["d"], cfg["L"], cfg["ff"]

    def linear(fan_in):
        return ("uniform", 1 / math.sqrt(fan_in))
    spec = [("tok", [V, d], ("uniform", 1)), ("pos", [T, d], ("uniform", 1))]
    for l in range(L):
        p = f"b{l}."
        spec += [(f"{p}ln1.g", [d], ("ones",)), (f"{p}ln1.b", [d], ("zeros",)),
                 (f"{p}wq", [d, d], linear(d)), (f"{p}wk", [d, d], linear(d)), (f"{p}wv", [d, d], linear(d)),
                 (f"{p}wo", [d, d], linear(d)), (f"{p}bo", [d], linear(d)),
                 (f"{p}ln2.g", [d], ("ones",)), (f"{p}ln2.b", [d], ("zeros",)),
                 (f"{p}w1", [d, ff], linear(d)), (f"{p}b1", [ff], linear(d)),
                 (f"{p}w2", [ff, d], linear(ff)), (f"{p}b2", [d], linear(ff))]
    spec += [("lnf.g", [d], ("ones",)), ("lnf.b", [d], ("zeros",)), ("head", [d, V], linear(d)),
             ("headb", [V], linear(d))]
    return spec


def _count(shape):
    n = 1
    for d in shape:
        n *= d
    return n


def param_count(V, cfg=CONFIG):
    return sum(_count(s) for _, s, _ in param_spec(V, cfg))


def init_params(V, seed, cfg=CONFIG):
    """Uniform initial parameters drawn in param_spec order (src/m3b/model.js:54-62)."""
    rng = Rng((seed * 7001 + 13) & 0xFFFFFFFF)
    out = {}
    for name, shape, init in param_spec(V, cfg):
        n = _count(shape)
        if init[0] == "uniform":
            b = init[1]
            out[name] = list(rng.uniform_array(n, -b, b))
        else:
            out[name] = [1.0 if init[0] == "ones" else 0.0] * n
    return out


def init_params_normal(V, seed, std, cfg=CONFIG):
    """N(0, std) weights, ones/zeros for LayerNorm, for the C5 workload (mulberry32 + Box-Muller)."""
    rng = Rng((seed * 7001 + 13) & 0xFFFFFFFF)
    out = {}
    for name, shape, init in param_spec(V, cfg):
        n = _count(shape)
        if init[0] == "uniform":
            out[name] = rng.normal_array(n, 0.0, std)
        else:
            out[name] = [1.0 if init[0] == "ones" else 0.0] * n
    return out


def causal_mask(T, mask=-1e4, bug=None):
    reach = 1 if bug == "mask-off-by-one" else 0
    return [0 if j <= i + reach else mask for i in range(T) for j in range(T)]


def layer_norm(g, x, gain, bias, cfg=CONFIG, bug=None):
    d, eps = cfg["d"], cfg["eps"]
    mean = g.div(g.sum(x, 1, True), g.const(d))
    xc = g.sub(x, mean)
    variance = g.div(g.sum(g.mul(xc, xc), 1, True), g.const(d - 1 if bug == "ln-divisor" else d))
    y = g.div(xc, g.sqrt(g.add(variance, g.const(1e-3 if bug == "ln-eps" else eps))))
    return g.add(g.mul(y, gain), bias)


def gelu(g, x):
    cube = g.mul(x, g.mul(x, x))
    inner = g.mul(g.const(math.sqrt(2 / math.pi)), g.add(x, g.mul(g.const(0.044715), cube)))
    return g.mul(g.mul(g.const(0.5), x), g.add(g.const(1), g.tanh(inner)))


def _attention(g, a, p, B, cfg, bug=None, trace=None):
    T, d, H, dh = cfg["T"], cfg["d"], cfg["H"], cfg["dh"]

    def heads(w):
        return g.transpose(g.reshape(g.matmul(a, p[w]), [B, T, H, dh]), [0, 2, 1, 3])
    q, k, v = heads("wq"), heads("wk"), heads("wv")
    s = g.matmul(q, g.transpose(k, [0, 1, 3, 2]))
    if bug != "scale-missing":
        s = g.mul(s, g.const(1 / math.sqrt(dh)))
    if trace is not None:
        trace.append(s)
    s = g.add(s, g.const(causal_mask(T, cfg["mask"], bug), [T, T]))
    probs = g.softmax(s, 2 if bug == "softmax-wrong-axis" else 3)
    o = g.matmul(probs, v)
    if bug == "merge-no-transpose":
        merged = g.reshape(o, [B * T, d])
    else:
        merged = g.reshape(g.transpose(o, [0, 2, 1, 3]), [B * T, d])
    return g.add(g.matmul(merged, p["wo"]), p["bo"])


def _shift_matrix(T):
    m = [0] * (T * T)
    for p in range(T):
        m[p * T + (p + 1) % T] = 1
    return m


BLOCK_KEYS = ("ln1.g", "ln1.b", "wq", "wk", "wv", "wo", "bo", "ln2.g", "ln2.b", "w1", "b1", "w2", "b2")


def logits_of(g, ids, V, B, cfg=CONFIG, bug=None, trace=None):
    """src/m3b/model.js:112-124."""
    T, d, L = cfg["T"], cfg["d"], cfg["L"]
    pos = ids["pos"]
    if bug == "position-off-by-one":
        pos = g.matmul(g.const(_shift_matrix(T), [T, T]), pos)
    h = g.reshape(g.add(g.reshape(g.matmul(ids["x"], ids["tok"]), [B, T, d]), pos), [B * T, d])
    for l in range(L):
        p = {k: ids[f"b{l}.{k}"] for k in BLOCK_KEYS}
        h = g.add(h, _attention(g, layer_norm(g, h, p["ln1.g"], p["ln1.b"], cfg, bug), p, B, cfg, bug, trace))
        m = layer_norm(g, h, p["ln2.g"], p["ln2.b"], cfg, bug)
        h = g.add(h, g.add(g.matmul(gelu(g, g.add(g.matmul(m, p["w1"]), p["b1"])), p["w2"]), p["b2"]))
    return g.add(g.matmul(layer_norm(g, h, ids["lnf.g"], ids["lnf.b"], cfg, bug), ids["head"]), ids["headb"])


def loss_of(g, logits, y, rows):
    logp = g.log_softmax(logits, 1)
    return g.div(g.neg(g.sum(g.sum(g.mul(y, logp), 1), 0)), g.const(rows))


def build_forward(V, B, cfg=CONFIG, bug=None):
    """src/m3b/model.js:133-145."""
    T = cfg["T"]
    g = Graph()
    ids = {name: g.input(name, shape) for name, shape, _ in param_spec(V, cfg)}
    ids["x"] = g.input("x", [B * T, V])
    ids["y"] = g.input("y", [B * T, V])
    scores = []
    logits = logits_of(g, ids, V, B, cfg, bug, scores)
    loss = loss_of(g, logits, ids["y"], B * T)
    return {"graph": g, "ids": ids, "logits": logits, "loss": loss, "scores": scores}


# ---------------------------------------------------------------- Adam (src/m3b/adam.js)
ADAM_3B = {"kind": "adam", "lr": 2e-3, "beta1": 0.9, "beta2": 0.999, "eps": 1e-8, "weightDecay": 0}


def adam_state_spec(names, shapes):
    out = []
    for p in names:
        out.append((f"{p}.m", shapes[p]))
        out.append((f"{p}.v", shapes[p]))
    out.append(("beta1Pow", []))
    out.append(("beta2Pow", []))
    return out


def adam_initial_state(names, shapes):
    return {name: [1.0 if name.endswith("Pow") else 0.0] * _count(shape) for name, shape in adam_state_spec(names, shapes)}


def adam_update(B, names, ids, grads, state, opt, sabotage=None):
    """src/m3b/adam.js:24-48 (PyTorch's order)."""
    c = B.const
    outputs = {}

    def decayed(p):
        if sabotage == "weight-decay-sign":
            return B.sub(grads[p], B.mul(c(opt["weightDecay"]), ids[p]))
        return B.add(grads[p], B.mul(c(opt["weightDecay"]), ids[p]))
    b1 = B.mul(state["beta1Pow"], c(opt["beta1"]))
    b2 = B.mul(state["beta2Pow"], c(opt["beta2"]))
    outputs["beta1Pow"] = b1
    outputs["beta2Pow"] = b2
    bc1 = B.sub(c(1), b1)
    bc2 = B.sub(c(1), b1 if sabotage == "adam-bias-correction" else b2)
    step_size = B.div(c(opt["lr"]), bc1)
    sqrt_bc2 = B.sqrt(bc2)
    for p in names:
        gp = decayed(p)
        m = B.add(B.mul(c(opt["beta1"]), state[f"{p}.m"]), B.mul(c(1 - opt["beta1"]), gp))
        v = B.add(B.mul(c(opt["beta2"]), state[f"{p}.v"]), B.mul(c(1 - opt["beta2"]), B.mul(gp, gp)))
        denom = B.add(B.div(B.sqrt(v), sqrt_bc2), c(opt["eps"]))
        outputs[p] = B.sub(ids[p], B.mul(step_size, B.div(m, denom)))
        outputs[f"{p}.m"] = m
        outputs[f"{p}.v"] = v
    return outputs


def param_names(V, cfg=CONFIG):
    return [n for n, _, _ in param_spec(V, cfg)]


def param_shapes(V, cfg=CONFIG):
    return {n: s for n, s, _ in param_spec(V, cfg)}


def build_step3b(V, B, cfg=CONFIG, opt=ADAM_3B, bug=None, rules=None):
    """Forward + grad + Adam as one graph (src/m3b/step.js:18-31)."""
    f = build_forward(V, B, cfg, bug)
    names = param_names(V, cfg)
    G = grad(f["graph"], [f["loss"]], [f["ids"][n] for n in names], rules=rules)
    g = G.graph
    grads = {n: G.grads[k] for k, n in enumerate(names)}
    state = {name: g.input(name, shape) for name, shape in adam_state_spec(names, param_shapes(V, cfg))}
    outputs = adam_update(g, names, f["ids"], grads, state, opt)
    inputs = {**{n: f["ids"][n] for n in names}, "x": f["ids"]["x"], "y": f["ids"]["y"], **state}
    return {"graph": g, "names": names, "stateNames": list(state), "loss": f["loss"], "logits": f["logits"],
            "grads": grads, "inputs": inputs, "outputs": outputs, "cotangent": G.cotangents[0]}


def build_grad3b(V, B, cfg=CONFIG):
    """Forward + grad only (no optimizer): the data-parallel split point (src/m3b/step.js:23)."""
    f = build_forward(V, B, cfg)
    names = param_names(V, cfg)
    G = grad(f["graph"], [f["loss"]], [f["ids"][n] for n in names])
    grads = {n: G.grads[k] for k, n in enumerate(names)}
    inputs = {**{n: f["ids"][n] for n in names}, "x": f["ids"]["x"], "y": f["ids"]["y"]}
    return {"graph": G.graph, "names": names, "loss": f["loss"], "logits": f["logits"], "grads": grads,
            "inputs": inputs, "outputs": dict(grads), "cotangent": G.cotangents[0]}


def build_adam_graph(V, cfg=CONFIG, opt=ADAM_3B):
    """Adam alone, its gradients as inputs named ``g:<param>`` (the graph after the allreduce)."""
    g = Graph()
    names = param_names(V, cfg)
    shapes = param_shapes(V, cfg)
    ids = {n: g.input(n, shapes[n]) for n in names}
    grads = {n: g.input(f"g:{n}", shapes[n]) for n in names}
    state = {name: g.input(name, shape) for name, shape in adam_state_spec(names, shapes)}
    outputs = adam_update(g, names, ids, grads, state, opt)
    inputs = {**ids, **{f"g:{n}": grads[n] for n in names}, **state}
    return {"graph": g, "names": names, "inputs": inputs, "outputs": outputs}


def encode_batch(seqs, V, T):
    """One-hot x, y [B*T, V] from T+1-token sequences (src/m3b/data.js:62-72), as numpy float32."""
    import numpy as np
    B = len(seqs)
    x = np.zeros((B * T, V), dtype=np.float32)
    y = np.zeros((B * T, V), dtype=np.float32)
    for b, s in enumerate(seqs):
        for t in range(T):
            x[b * T + t, s[t]] = 1
            y[b * T + t, s[t + 1]] = 1
    return x, y
