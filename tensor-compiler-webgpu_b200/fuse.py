"""The fusion pass: replaces groups of nodes by one ``fused`` node each.

Restates ``src/fusion/fuse.js`` (``grow`` :54-169, ``label`` :172-180, ``body``
:183-199, ``fuse`` :215-292, ``fusionSummary`` :333-338).  The pass is the API
the backend consumes: it decides which fused nodes exist, and the backend
instantiates one CUDA template per fused node.  Grouping depends on iteration
order, so every set here is insertion-ordered (a ``dict``), as JavaScript's
``Set`` is, and every loop walks in the reference's order.

Kinds: ``elementwise`` (one element count, indexed loads through
broadcast/reshape/transpose), ``epilogue`` (a matmul whose only consumer is
such a group), ``rowwise`` (last-axis keepDims sum/max brought back by
broadcast: LayerNorm, softmax, ...).
"""
from __future__ import annotations

import copy
import math

from .ir import Graph, Node, size, same_shape, f32

ELEMENTWISE = frozenset(("add", "sub", "mul", "div", "neg", "exp", "log", "relu", "tanh", "sqrt", "step", "stopGradient"))
MOVES = frozenset(("broadcast", "reshape", "transpose"))
MAX_OPERANDS = 6
PATTERNS = ("elementwise", "epilogue", "rowwise")


def scalar_const(node):
    """A const holding one value whatever its shape (src/fusion/fuse.js:27-34)."""
    if node.op != "const":
        return False
    v = node.attrs["value"]
    first = v if isinstance(v, (int, float)) else v[0]
    if not math.isfinite(f32(float(first))):
        return False
    return isinstance(v, (int, float)) or all(_same_value(x, first) for x in v)


def _same_value(a, b):
    # Object.is: distinguishes -0 from 0, equates NaN with NaN
    a, b = float(a), float(b)
    if math.isnan(a) and math.isnan(b):
        return True
    return a == b and math.copysign(1.0, a) == math.copysign(1.0, b)


def const_value(node):
    v = node.attrs["value"]
    return v if isinstance(v, (int, float)) else v[0]


def consumers_of(graph):
    c = [[] for _ in graph.nodes]
    for n in graph.nodes:
        for i in dict.fromkeys(n.inputs):
            c[i].append(n.id)
    return c


def _last_axis_reduce(graph, n):
    return n.op in ("sum", "max") and n.attrs.get("keepDims") and \
        n.attrs["axis"] == len(graph.nodes[n.inputs[0]].shape) - 1


def _row_shape(s):
    return list(s[:-1]) + [1]


def _grow(graph, sink, consumers, taken, keep, patterns, recompute, max_operands, sabotage):
    nodes = graph.nodes
    S = nodes[sink].shape
    n = size(S)
    members = {sink: None}
    state = {"kind": "elementwise", "root": None}
    C = S[-1] if S else 1

    def is_row_shape(s):
        return len(s) == len(S) and same_shape(s, _row_shape(S))

    def free(i):
        return i not in taken or recompute

    def all_in(i, extra=()):
        return all(c in members or c in extra for c in consumers[i])

    def exclusive(i, extra=()):
        return i not in keep and (recompute or all_in(i, extra) or sabotage == "fusion-absorbs-shared")

    def operands_of(s):
        ext = {}
        for m in s:
            node = nodes[m]
            if node.op == "const":
                continue
            for i in node.inputs:
                if i not in s:
                    ext[i] = None
        return ext

    def fits(s):
        return len(operands_of(s)) <= max_operands

    def row_region(b):
        region = {}
        reductions = 0
        stack = [nodes[b].inputs[0]]
        while stack:
            i = stack.pop()
            if i in region or i in members:
                continue
            node = nodes[i]
            if scalar_const(node):
                region[i] = None
                continue
            if node.op == "broadcast" and scalar_const(nodes[node.inputs[0]]):
                region[i] = None
                region[node.inputs[0]] = None
                continue
            if not is_row_shape(node.shape) or not free(i):
                continue
            if _last_axis_reduce(graph, node) and same_shape(nodes[node.inputs[0]].shape, S):
                region[i] = None
                reductions += 1
                continue
            if node.op in ELEMENTWISE or node.op == "stopGradient":
                region[i] = None
                stack.extend(node.inputs)
        if not reductions:
            return None
        extra = dict(region)
        extra[b] = None
        for i in region:
            if not scalar_const(nodes[i]) and nodes[i].op != "broadcast" and not exclusive(i, extra):
                return None
        return region

    def try_add(items):
        nxt = dict(members)
        for i in items:
            nxt[i] = None
        if not fits(nxt):
            return False
        for i in items:
            members[i] = None
        return True

    changed = True
    while changed:
        changed = False
        for m in list(members):
            m_node = nodes[m]
            if m_node.op == "const" or m == state["root"] or m_node.op in ("broadcast", "transpose"):
                continue
            row_tier = state["kind"] == "rowwise" and not _last_axis_reduce(graph, m_node) and \
                m_node.op != "broadcast" and is_row_shape(m_node.shape)
            for p in dict.fromkeys(m_node.inputs):
                if p in members:
                    continue
                if state["root"] is not None and p in nodes[state["root"]].inputs:
                    continue
                pn = nodes[p]
                if scalar_const(pn):
                    changed = try_add([p]) or changed
                    continue
                if pn.op == "broadcast" and scalar_const(nodes[pn.inputs[0]]):
                    changed = try_add([p, pn.inputs[0]]) or changed
                    continue
                if not free(p) or not exclusive(p):
                    continue
                if pn.op in ELEMENTWISE or pn.op == "reshape":
                    changed = try_add([p]) or changed
                    continue
                if pn.op in ("broadcast", "transpose") and m_node.op not in ("broadcast", "transpose"):
                    src = nodes[pn.inputs[0]]
                    if (pn.op == "broadcast" and "rowwise" in patterns and state["root"] is None and not row_tier
                            and same_shape(pn.shape, S) and is_row_shape(src.shape) and C > 1):
                        region = row_region(p)
                        if region is not None and try_add([p] + list(region)):
                            state["kind"] = "rowwise"
                            changed = True
                            continue
                    if recompute and state["kind"] != "rowwise" and src.op in ELEMENTWISE and free(src.id) \
                            and src.id not in keep:
                        if try_add([p, src.id]):
                            changed = True
                            continue
                    changed = try_add([p]) or changed
                    continue
                if (pn.op == "matmul" and "epilogue" in patterns and state["kind"] == "elementwise"
                        and state["root"] is None and size(pn.shape) == n and not row_tier
                        and not any(i in members for i in pn.inputs)):
                    if try_add([p]):
                        state["kind"] = "epilogue"
                        state["root"] = p
                        changed = True
                    continue
    if state["kind"] == "elementwise" and "elementwise" not in patterns:
        return None
    real = [i for i in members if nodes[i].op != "const"]
    if len(real) < 2:
        return None
    return members, state["kind"], state["root"]


def _label(graph, members, kind):
    """src/fusion/fuse.js:172-180."""
    if kind != "rowwise":
        return "matmul-epilogue" if kind == "epilogue" else "elementwise"
    ops = [graph.nodes[i].op for i in members]

    def count(op):
        return sum(1 for o in ops if o == op)
    if count("sum") >= 2 and count("sqrt") >= 1:
        return "layernorm"
    if count("max") >= 1 and count("exp") >= 1 and count("sum") >= 1 and count("log") >= 1:
        return "log-softmax"
    if count("max") >= 1 and count("exp") >= 1 and count("sum") >= 1 and count("div") >= 1:
        return "softmax"
    return "rowwise"


def _body(graph, members, sink):
    """Body graph of a group: inputs a0.. for operands, then members in id order."""
    g = Graph()
    operands = []
    mapping = {}
    for i in sorted(members):
        node = graph.nodes[i]
        for j in node.inputs:
            if j not in members and j not in mapping:
                mapping[j] = g.input(f"a{len(operands)}", graph.nodes[j].shape)
                operands.append(j)
        mapping[i] = g.emit(node.op, [mapping[j] for j in node.inputs], node.attrs)
    return g, operands, mapping[sink]


class Group:
    __slots__ = ("sink", "members", "kind", "root", "pattern")

    def __init__(self, sink, members, kind, root, pattern):
        self.sink, self.members, self.kind, self.root, self.pattern = sink, members, kind, root, pattern


class FuseResult:
    __slots__ = ("graph", "origin", "index", "groups")

    def __init__(self, graph, origin, index, groups):
        self.graph, self.origin, self.index, self.groups = graph, origin, index, groups


def fuse(graph, patterns=PATTERNS, recompute=False, keep=(), max_operands=MAX_OPERANDS, sabotage=None):
    """Fuse ``graph`` (src/fusion/fuse.js:215-292).

    Returns ``FuseResult(graph, origin, index, groups)``: ``origin[new] = old``
    and ``index[old] = new`` for every surviving node.
    """
    nodes = graph.nodes
    consumers = consumers_of(graph)
    keep_set = set(keep)
    taken = set()
    groups = []
    sink_of = {}
    for nid in range(len(nodes) - 1, -1, -1):
        node = nodes[nid]
        if nid in taken or node.op not in ELEMENTWISE:
            continue
        gr = _grow(graph, nid, consumers, taken, keep_set, patterns, recompute, max_operands, sabotage)
        if gr is None:
            continue
        members, kind, root = gr
        for m in members:
            mn = nodes[m]
            if mn.op != "const" and not (mn.op == "broadcast" and scalar_const(nodes[mn.inputs[0]])):
                taken.add(m)
        group = Group(nid, members, kind, root, _label(graph, members, kind))
        groups.append(group)
        sink_of[nid] = group

    rewire = {}
    if sabotage == "fusion-absorbs-shared":
        for gr in groups:
            for m in gr.members:
                if m == gr.sink or nodes[m].op == "const":
                    continue
                if any(c not in gr.members for c in consumers[m]):
                    rewire[m] = gr.sink

    def via(i):
        return rewire.get(i, i)

    needed = set()
    built = {}
    for nid in range(len(nodes) - 1, -1, -1):
        node = nodes[nid]
        if not consumers[nid] or nid in keep_set:
            needed.add(nid)
        if nid not in needed:
            continue
        if nid in sink_of:
            b = _body(graph, sink_of[nid].members, nid)
            built[nid] = b
            for o in b[1]:
                needed.add(via(o))
        else:
            for i in node.inputs:
                needed.add(via(i))

    out = Graph()
    index = {}
    origin = []

    def ref(i):
        r = via(i)
        if r not in index:
            raise RuntimeError(f"fuse: node {r} used before it is built")
        return index[r]

    for node in nodes:
        if node.id not in needed:
            continue
        if node.id in built:
            gr = sink_of[node.id]
            bg, operands, output = built[node.id]
            new_id = len(out.nodes)
            out.nodes.append(Node(new_id, "fused", [ref(o) for o in operands],
                                  {"kind": gr.kind, "pattern": gr.pattern, "body": bg.to_json(), "output": output},
                                  list(node.shape)))
        elif rewire and node.op not in ("input", "const"):
            new_id = len(out.nodes)
            out.nodes.append(Node(new_id, node.op, [ref(i) for i in node.inputs], copy.deepcopy(node.attrs),
                                  list(node.shape)))
        else:
            new_id = out.emit(node.op, [ref(i) for i in node.inputs], node.attrs)
        index[node.id] = new_id
        origin.append(node.id)
    return FuseResult(out, origin, index, groups)


_bodies = {}


def body_of(node):
    """The body of a fused node as a Graph (cached by node identity)."""
    key = id(node.attrs["body"])
    hit = _bodies.get(key)
    if hit is None or hit[0] is not node.attrs["body"]:
        hit = (node.attrs["body"], Graph.from_json(node.attrs["body"]))
        _bodies[key] = hit
    return hit[1]


def fusion_summary(original, fused):
    """Launch counts before/after and fused nodes by pattern (src/fusion/fuse.js:333-338)."""
    def launches(g):
        return sum(1 for n in g.nodes if n.op not in ("input", "const"))
    by = {}
    for n in fused.graph.nodes:
        if n.op == "fused":
            by[n.attrs["pattern"]] = by.get(n.attrs["pattern"], 0) + 1
    return {"launchesBefore": launches(original), "launchesAfter": launches(fused.graph), "byPattern": by}
