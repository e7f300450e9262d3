"""The tensor IR: an SSA node list with shapes inferred at creation.

Host-side restatement of the reference's IR so the backend can be driven
without a JavaScript engine.  Semantics follow ``src/ir/graph.js`` (builder,
``emit``, composites) and ``src/ir/shapes.js`` (shape rules, broadcasting).
Node ids are list positions, so a graph is always in topological order.

Interchange is the reference's ``Graph.toJSON`` form
(``{"nodes": [{op, inputs, attrs, shape}]}``, src/ir/graph.js:48-50), so
graphs written by the reference (golden/cases.json) load unchanged.
"""
from __future__ import annotations

import copy
import math

UNARY = ("neg", "exp", "log", "relu", "tanh", "step", "stopGradient", "sqrt")
BINARY = ("add", "sub", "mul", "div")
REDUCE = ("sum", "max")
# src/ir/shapes.js:51-52 (same order)
OPS = ("input", "const") + BINARY + UNARY + ("matmul",) + REDUCE + ("broadcast", "reshape", "transpose")


class ShapeError(ValueError):
    """A shape rule was broken (src/ir/shapes.js:3-5)."""


def size(shape):
    n = 1
    for d in shape:
        n *= d
    return n


def same_shape(a, b):
    return len(a) == len(b) and all(x == y for x, y in zip(a, b))


def fmt(shape):
    return "[" + ",".join(str(d) for d in shape) + "]"


def _is_int(v):
    return isinstance(v, int) and not isinstance(v, bool)


def check_shape(shape, what):
    if not isinstance(shape, (list, tuple)) or not all(_is_int(d) and d >= 1 for d in shape):
        raise ShapeError(f"{what}: shape must be a list of positive integers, got {shape!r}")


def norm_axis(axis, rank, op):
    """src/ir/shapes.js:17-24."""
    a = axis + rank if axis < 0 else axis
    if not _is_int(a) or a < 0 or a >= rank:
        raise ShapeError(f"{op}: axis {axis} out of range for rank {rank}")
    return a


def broadcast_shapes(a, b):
    """NumPy broadcasting of two shapes, or None (src/ir/shapes.js:27-37)."""
    rank = max(len(a), len(b))
    out = []
    for i in range(rank):
        ia = len(a) - rank + i
        ib = len(b) - rank + i
        da = a[ia] if ia >= 0 else 1
        db = b[ib] if ib >= 0 else 1
        if da != db and da != 1 and db != 1:
            return None
        out.append(max(da, db))
    return out


def broadcasts_to(frm, to):
    """src/ir/shapes.js:40-44."""
    if len(frm) > len(to):
        return False
    lead = len(to) - len(frm)
    return all(d == 1 or d == to[lead + i] for i, d in enumerate(frm))


def infer_shape(op, shapes, attrs):
    """The result shape of ``op`` (src/ir/shapes.js:55-114)."""
    if op not in OPS:
        raise ShapeError(f"unknown op '{op}'")
    want = {"input": 0, "const": 0, "matmul": 2}.get(op, 2 if op in BINARY else 1)
    if len(shapes) != want:
        raise ShapeError(f"{op}: takes {want} inputs, got {len(shapes)}")
    if op in ("input", "const"):
        check_shape(attrs.get("shape"), op)
        if op == "const":
            v = attrs.get("value")
            ok = isinstance(v, (int, float)) and not isinstance(v, bool) or (
                isinstance(v, (list, tuple)) and len(v) == size(attrs["shape"]))
            if not ok:
                raise ShapeError(f"const: value must be a number or {size(attrs['shape'])} numbers")
        return list(attrs["shape"])
    if op in BINARY:
        if not same_shape(shapes[0], shapes[1]):
            raise ShapeError(f"{op}: shapes {fmt(shapes[0])} and {fmt(shapes[1])} differ; broadcast explicitly")
        return list(shapes[0])
    if op in UNARY:
        return list(shapes[0])
    if op == "matmul":
        a, b = shapes
        if len(a) < 2 or len(b) < 2:
            raise ShapeError(f"matmul: needs rank >= 2, got {fmt(a)} and {fmt(b)}")
        if len(a) != len(b) or not same_shape(a[:-2], b[:-2]):
            raise ShapeError(f"matmul: batch dims of {fmt(a)} and {fmt(b)} differ")
        if a[-1] != b[-2]:
            raise ShapeError(f"matmul: inner dims of {fmt(a)} and {fmt(b)} differ")
        return list(a[:-1]) + [b[-1]]
    if op in REDUCE:
        x = shapes[0]
        axis = norm_axis(attrs["axis"], len(x), op)
        if attrs["axis"] != axis:
            raise ShapeError(f"{op}: axis must be stored normalised")
        if attrs.get("keepDims"):
            return [1 if i == axis else d for i, d in enumerate(x)]
        return [d for i, d in enumerate(x) if i != axis]
    if op == "broadcast":
        check_shape(attrs.get("shape"), op)
        if not broadcasts_to(shapes[0], attrs["shape"]):
            raise ShapeError(f"broadcast: {fmt(shapes[0])} does not broadcast to {fmt(attrs['shape'])}")
        return list(attrs["shape"])
    if op == "reshape":
        check_shape(attrs.get("shape"), op)
        if size(attrs["shape"]) != size(shapes[0]):
            raise ShapeError(f"reshape: {fmt(shapes[0])} has {size(shapes[0])} elements, "
                             f"{fmt(attrs['shape'])} has {size(attrs['shape'])}")
        return list(attrs["shape"])
    if op == "transpose":
        x = shapes[0]
        p = attrs.get("perm")
        ok = isinstance(p, (list, tuple)) and len(p) == len(x) and sorted(p) == list(range(len(x)))
        if not ok:
            raise ShapeError(f"transpose: {p!r} is not a permutation of rank {len(x)}")
        return [x[i] for i in p]
    raise ShapeError(f"no shape rule for '{op}'")


class Node:
    __slots__ = ("id", "op", "inputs", "attrs", "shape")

    def __init__(self, id, op, inputs, attrs, shape):
        self.id = id
        self.op = op
        self.inputs = inputs
        self.attrs = attrs
        self.shape = shape

    def __repr__(self):
        return f"Node({self.id}, {self.op}, {self.inputs}, {fmt(self.shape)})"


class Graph:
    """src/ir/graph.js:15-147: raw ``emit`` plus a broadcasting builder."""

    def __init__(self):
        self.nodes = []

    def emit(self, op, inputs=(), attrs=None):
        attrs = {} if attrs is None else attrs
        for i in inputs:
            if not _is_int(i) or i < 0 or i >= len(self.nodes):
                raise ShapeError(f"{op}: input {i} is not a value of this graph")
        shape = infer_shape(op, [self.nodes[i].shape for i in inputs], attrs)
        nid = len(self.nodes)
        self.nodes.append(Node(nid, op, list(inputs), copy.deepcopy(attrs), shape))
        return nid

    def shape(self, nid):
        return self.nodes[nid].shape

    def input_id(self, name):
        for n in self.nodes:
            if n.op == "input" and n.attrs["name"] == name:
                return n.id
        return None

    def inputs(self):
        return [n for n in self.nodes if n.op == "input"]

    def clone(self):
        g = Graph()
        g.nodes = [Node(n.id, n.op, list(n.inputs), copy.deepcopy(n.attrs), list(n.shape)) for n in self.nodes]
        return g

    def to_json(self):
        return {"nodes": [{"op": n.op, "inputs": list(n.inputs), "attrs": copy.deepcopy(n.attrs),
                           "shape": list(n.shape)} for n in self.nodes]}

    @staticmethod
    def from_json(js):
        g = Graph()
        for n in js["nodes"]:
            nid = g.emit(n["op"], n["inputs"], n["attrs"])
            if not same_shape(g.shape(nid), n["shape"]):
                raise ShapeError(f"node {nid}: stored shape {fmt(n['shape'])} but inferred {fmt(g.shape(nid))}")
        return g

    # ---- builder (src/ir/graph.js:66-128) ----
    def input(self, name, shape):
        if self.input_id(name) is not None:
            raise ValueError(f"input '{name}' already exists")
        return self.emit("input", [], {"name": name, "shape": list(shape)})

    def const(self, value, shape=()):
        return self.emit("const", [], {"shape": list(shape), "value": value})

    def broadcast(self, x, shape):
        return x if same_shape(self.shape(x), shape) else self.emit("broadcast", [x], {"shape": list(shape)})

    def _binary(self, op, a, b):
        shape = broadcast_shapes(self.shape(a), self.shape(b))
        if shape is None:
            raise ShapeError(f"{op}: {fmt(self.shape(a))} and {fmt(self.shape(b))} do not broadcast")
        return self.emit(op, [self.broadcast(a, shape), self.broadcast(b, shape)])

    def add(self, a, b): return self._binary("add", a, b)
    def sub(self, a, b): return self._binary("sub", a, b)
    def mul(self, a, b): return self._binary("mul", a, b)
    def div(self, a, b): return self._binary("div", a, b)
    def neg(self, x): return self.emit("neg", [x])
    def exp(self, x): return self.emit("exp", [x])
    def log(self, x): return self.emit("log", [x])
    def relu(self, x): return self.emit("relu", [x])
    def tanh(self, x): return self.emit("tanh", [x])
    def sqrt(self, x): return self.emit("sqrt", [x])
    def step(self, x): return self.emit("step", [x])
    def stop_gradient(self, x): return self.emit("stopGradient", [x])
    def matmul(self, a, b): return self.emit("matmul", [a, b])

    def sum(self, x, axis, keep_dims=False):
        return self.emit("sum", [x], {"axis": norm_axis(axis, len(self.shape(x)), "sum"), "keepDims": keep_dims})

    def max(self, x, axis, keep_dims=False):
        return self.emit("max", [x], {"axis": norm_axis(axis, len(self.shape(x)), "max"), "keepDims": keep_dims})

    def reshape(self, x, shape):
        return x if same_shape(self.shape(x), shape) else self.emit("reshape", [x], {"shape": list(shape)})

    def transpose(self, x, perm=None):
        rank = len(self.shape(x))
        if perm is None:
            perm = list(range(rank))[::-1]
        if all(p == i for i, p in enumerate(perm)):
            return x
        return self.emit("transpose", [x], {"perm": list(perm)})

    def transpose_last2(self, x):
        rank = len(self.shape(x))
        perm = list(range(rank))
        perm[rank - 2], perm[rank - 1] = perm[rank - 1], perm[rank - 2]
        return self.transpose(x, perm)

    # ---- composites (src/ir/graph.js:132-146) ----
    def _shifted(self, x, axis):
        m = self.stop_gradient(self.max(x, axis, True))
        return self.sub(x, m)

    def softmax(self, x, axis=-1):
        z = self.exp(self._shifted(x, axis))
        return self.div(z, self.sum(z, axis, True))

    def log_softmax(self, x, axis=-1):
        z = self._shifted(x, axis)
        return self.sub(z, self.log(self.sum(self.exp(z), axis, True)))


def strides(shape):
    """Row-major strides (src/interp.js:9-14)."""
    s = [0] * len(shape)
    acc = 1
    for i in range(len(shape) - 1, -1, -1):
        s[i] = acc
        acc *= shape[i]
    return s


def f32(v):
    """Round a Python float to the nearest float32 value (Math.fround)."""
    import struct
    if math.isnan(v):
        return v
    try:
        return struct.unpack("f", struct.pack("f", v))[0]
    except OverflowError:
        return math.copysign(math.inf, v)
