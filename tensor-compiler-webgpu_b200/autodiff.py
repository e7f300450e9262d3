"""Reverse-mode autodiff as a graph-to-graph transform.

Restates ``src/autodiff.js``: the rule table ``RULES`` (src/autodiff.js:25-76)
and ``grad`` (src/autodiff.js:87-127).  The gradient graph is an ordinary graph
(the forward nodes keep their ids), so the same fusion pass and backend run it.
"""
from __future__ import annotations

from .ir import same_shape


class GradientError(ValueError):
    pass


def _mul_rule(G, n, gy):
    a, b = n.inputs
    return [G.mul(gy, b), G.mul(gy, a)]


def _div_rule(G, n, gy):
    a, b = n.inputs
    return [G.div(gy, b), G.neg(G.div(G.mul(gy, a), G.mul(b, b)))]


def _matmul_rule(G, n, gy):
    a, b = n.inputs
    return [G.matmul(gy, G.transpose_last2(b)), G.matmul(G.transpose_last2(a), gy)]


def _sum_rule(G, n, gy):
    x = n.inputs[0]
    xs = G.shape(x)
    kept = [1 if i == n.attrs["axis"] else d for i, d in enumerate(xs)]
    return [G.broadcast(G.reshape(gy, kept), xs)]


def _broadcast_rule(G, n, gy):
    xs = G.shape(n.inputs[0])
    lead = len(n.shape) - len(xs)
    g = gy
    for _ in range(lead):          # axes added in front: summed away
        g = G.sum(g, 0, False)
    for i, d in enumerate(xs):     # axes stretched from 1: summed, kept
        if d == 1 and n.shape[lead + i] != 1:
            g = G.sum(g, i, True)
    return [G.reshape(g, xs)]


def _transpose_rule(G, n, gy):
    perm = n.attrs["perm"]
    inverse = [0] * len(perm)
    for i, p in enumerate(perm):
        inverse[p] = i
    return [G.transpose(gy, inverse)]


def _max_rule(G, n, gy):
    raise GradientError("max has no gradient; wrap it in stopGradient where its gradient is zero (as softmax does)")


RULES = {
    "add": lambda G, n, gy: [gy, gy],
    "sub": lambda G, n, gy: [gy, G.neg(gy)],
    "mul": _mul_rule,
    "div": _div_rule,
    "neg": lambda G, n, gy: [G.neg(gy)],
    "exp": lambda G, n, gy: [G.mul(gy, n.id)],
    "log": lambda G, n, gy: [G.div(gy, n.inputs[0])],
    "relu": lambda G, n, gy: [G.mul(gy, G.step(n.inputs[0]))],
    "tanh": lambda G, n, gy: [G.mul(gy, G.sub(G.const(1), G.mul(n.id, n.id)))],
    "sqrt": lambda G, n, gy: [G.div(gy, G.mul(G.const(2), n.id))],
    "matmul": _matmul_rule,
    "sum": _sum_rule,
    "broadcast": _broadcast_rule,
    "reshape": lambda G, n, gy: [G.reshape(gy, G.shape(n.inputs[0]))],
    "transpose": _transpose_rule,
    "step": lambda G, n, gy: [None],
    "stopGradient": lambda G, n, gy: [None],
    "max": _max_rule,
}


class GradResult:
    __slots__ = ("graph", "cotangents", "grads")

    def __init__(self, graph, cotangents, grads):
        self.graph = graph
        self.cotangents = cotangents
        self.grads = grads


def grad(graph, outputs, wrt, rules=None, prefix="d"):
    """The gradient graph of ``graph`` (src/autodiff.js:87-127).

    Returns ``GradResult(graph, cotangents, grads)``: cotangent input names per
    output and the gradient node id per ``wrt`` entry.
    """
    rules = RULES if rules is None else rules
    G = graph.clone()
    forward_count = len(graph.nodes)
    depends = [False] * forward_count
    for i in wrt:
        depends[i] = True
    for node in graph.nodes:
        if any(depends[i] for i in node.inputs):
            depends[node.id] = True

    cot = [None] * forward_count

    def accumulate(nid, contribution):
        if not same_shape(G.shape(contribution), graph.nodes[nid].shape):
            raise GradientError(f"gradient for node {nid} has shape {G.shape(contribution)}, "
                                f"value has {graph.nodes[nid].shape}")
        cot[nid] = contribution if cot[nid] is None else G.add(cot[nid], contribution)

    cotangents = []
    for i, oid in enumerate(outputs):
        name = f"{prefix}{i}"
        accumulate(oid, G.input(name, graph.nodes[oid].shape))
        cotangents.append(name)

    for nid in range(forward_count - 1, -1, -1):
        node = graph.nodes[nid]
        if cot[nid] is None or not depends[nid] or not node.inputs:
            continue
        if not any(depends[i] for i in node.inputs):
            continue
        rule = rules.get(node.op)
        if rule is None:
            raise GradientError(f"no gradient rule for '{node.op}'")
        contributions = rule(G, node, cot[nid])
        for k, inp in enumerate(node.inputs):
            if contributions[k] is not None and depends[inp]:
                accumulate(inp, contributions[k])

    grads = [cot[i] if cot[i] is not None else G.const(0, list(graph.nodes[i].shape)) for i in wrt]
    return GradResult(G, cotangents, grads)
