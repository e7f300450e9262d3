"""ORACLE -- test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may
import this module; the product path never does.  It wraps ``liboracle.so``
(``interp.c``: the C restatement of src/interp.js and src/gpu/bounds.js) and
restates the reference's judging helpers:

* ``evaluate``            src/interp.js:136-157 (float64, index order)
* ``reference_with_bounds`` src/gpu/bounds.js:91-136 (amendment 8, S = 2)
* ``evaluate_fused`` / ``check_semantics`` src/fusion/fuse.js:295-330
* ``judge``               src/gpu/bounds.js:155-171
* ``judge_fused``         src/gpu/harness-m4.js:46-60
* ``local_reference_fused`` src/gpu/harness-m4.js:182-200
* ``judge_outputs``       src/fusion/workloads.js:351-367 (the 1% unjudgeable rule)
* ``tensor_score``        src/testing/golden.js:36-49 (metric v2, 1e-12)
"""
from __future__ import annotations

import ctypes
import importlib
import math
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

S = 2
F32_MAX = 3.4028234663852886e38
MAX_RANK = 8
OPCODE = {"input": 0, "const": 1, "add": 2, "sub": 3, "mul": 4, "div": 5, "neg": 6, "exp": 7, "log": 8, "relu": 9,
          "tanh": 10, "step": 11, "stopGradient": 12, "sqrt": 13, "matmul": 14, "sum": 15, "max": 16,
          "broadcast": 17, "reshape": 18, "transpose": 19}


def _pkg():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    return importlib.import_module("tensor-compiler-webgpu_b200")


class _Node(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int32), ("n_in", ctypes.c_int32), ("in0", ctypes.c_int32), ("in1", ctypes.c_int32),
                ("rank", ctypes.c_int32), ("axis", ctypes.c_int32), ("keep_dims", ctypes.c_int32),
                ("pad", ctypes.c_int32), ("shape", ctypes.c_int64 * MAX_RANK), ("perm", ctypes.c_int32 * MAX_RANK),
                ("data", ctypes.c_void_p), ("scalar", ctypes.c_double), ("data_bound", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("out_bound", ctypes.c_void_p)]


def build(force=False):
    """Compile liboracle.so (gcc -O2, no SIMD intrinsics, no threads)."""
    src = os.path.join(HERE, "interp.c")
    if not force and os.path.exists(LIB_PATH) and os.path.getmtime(LIB_PATH) >= max(
            os.path.getmtime(src), os.path.getmtime(os.path.join(HERE, "interp.h"))):
        return LIB_PATH
    subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.tco_evaluate.argtypes = [ctypes.POINTER(_Node), ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
        _lib.tco_evaluate.restype = ctypes.c_int
    return _lib


def _size(shape):
    n = 1
    for d in shape:
        n *= d
    return n


def _f64(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64).reshape(-1))


def _run(graph, inputs, with_bounds, want=None, carried=None):
    """Evaluate ``graph``; returns (values, bounds) lists (None where not wanted)."""
    nodes = graph.nodes
    n = len(nodes)
    arr = (_Node * max(n, 1))()
    keep = []  # keeps numpy buffers alive
    values = [None] * n
    bounds = [None] * n
    want = set(range(n)) if want is None else set(want)
    carried = carried or {}
    for node in nodes:
        c = arr[node.id]
        c.op = OPCODE[node.op]
        c.n_in = len(node.inputs)
        c.in0 = node.inputs[0] if node.inputs else -1
        c.in1 = node.inputs[1] if len(node.inputs) > 1 else -1
        if len(node.shape) > MAX_RANK:
            raise ValueError("rank too large for the oracle")
        c.rank = len(node.shape)
        for i, d in enumerate(node.shape):
            c.shape[i] = d
        if node.op in ("sum", "max"):
            c.axis = node.attrs["axis"]
            c.keep_dims = 1 if node.attrs.get("keepDims") else 0
        if node.op == "transpose":
            for i, p in enumerate(node.attrs["perm"]):
                c.perm[i] = p
        if node.op == "input":
            name = node.attrs["name"]
            if name in carried:
                v, b = carried[name]
                v, b = _f64(v), _f64(b)
                if v.size != _size(node.shape):
                    raise ValueError(f"carried input '{name}' has {v.size} values, needs {_size(node.shape)}")
                keep += [v, b]
                c.data = v.ctypes.data
                c.data_bound = b.ctypes.data
            else:
                if name not in inputs:
                    raise KeyError(f"no value for input '{name}'")
                v = _f64(inputs[name])
                if v.size != _size(node.shape):
                    raise ValueError(f"input '{name}': expected {_size(node.shape)} numbers, got {v.size}")
                keep.append(v)
                c.data = v.ctypes.data
        elif node.op == "const":
            val = node.attrs["value"]
            if isinstance(val, (int, float)):
                c.data = None
                c.scalar = float(val)
            else:
                v = _f64(val)
                keep.append(v)
                c.data = v.ctypes.data
        if node.id in want:
            o = np.empty(max(1, _size(node.shape)), dtype=np.float64)
            values[node.id] = o[:_size(node.shape)]
            keep.append(o)
            c.out = o.ctypes.data
            if with_bounds:
                ob = np.empty(max(1, _size(node.shape)), dtype=np.float64)
                bounds[node.id] = ob[:_size(node.shape)]
                keep.append(ob)
                c.out_bound = ob.ctypes.data
    err = ctypes.create_string_buffer(512)
    rc = lib().tco_evaluate(arr, n, 1 if with_bounds else 0, err, 512)
    if rc != 0:
        raise RuntimeError(f"oracle: {err.value.decode()}")
    return values, bounds


def evaluate(graph, inputs, want=None):
    """float64 value of every node (src/interp.js:136-157); fused nodes are evaluated through their bodies."""
    if any(n.op == "fused" for n in graph.nodes):
        return evaluate_fused(graph, inputs)
    return _run(graph, inputs, False, want)[0]


def reference_with_bounds(graph, inputs, carried=None, want=None):
    """(values, bounds, rounded inputs) as src/gpu/bounds.js:91-136 computes them."""
    values, bounds = _run(graph, inputs, True, want, carried)
    rounded = {}
    for node in graph.nodes:
        if node.op == "input":
            name = node.attrs["name"]
            if carried and name in carried:
                rounded[name] = _f64(carried[name][0])
            else:
                rounded[name] = _f64(inputs[name]).astype(np.float32).astype(np.float64)
    return values, bounds, rounded


def evaluate_fused(graph, inputs):
    """FUSED_KERNELS semantics: a fused node is its body evaluated on its operands (fuse.js:295-305)."""
    pkg = _pkg()
    vals = [None] * len(graph.nodes)
    for node in graph.nodes:
        if node.op == "input":
            vals[node.id] = _f64(inputs[node.attrs["name"]])
            continue
        if node.op == "fused":
            body = pkg.fuse.body_of(node)
            feed = {f"a{k}": vals[i] for k, i in enumerate(node.inputs)}
            vals[node.id] = _run(body, feed, False, [node.attrs["output"]])[0][node.attrs["output"]]
            continue
        g = pkg.ir.Graph()
        ins = [g.input(f"a{k}", graph.nodes[i].shape) for k, i in enumerate(node.inputs)]
        if node.op == "const":
            out = g.emit("const", [], node.attrs)
        else:
            out = g.emit(node.op, ins, node.attrs)
        feed = {f"a{k}": vals[i] for k, i in enumerate(node.inputs)}
        vals[node.id] = _run(g, feed, False, [out])[0][out]
    return vals


def check_semantics(original, fused, inputs):
    """Bitwise float64 equality at every surviving node (src/fusion/fuse.js:311-330)."""
    a = evaluate(original, inputs)
    try:
        b = evaluate_fused(fused.graph, inputs)
    except Exception as exc:  # the sabotaged pass may build an invalid graph
        return {"identical": False, "compared": 0, "first": {"error": str(exc)}}
    compared = 0
    for nid in range(len(fused.graph.nodes)):
        o = fused.origin[nid]
        x, y = a[o], b[nid]
        if x.size != y.size:
            return {"identical": False, "compared": compared, "first": {"node": nid, "origin": o, "reason": "length"}}
        same = (x.view(np.uint64) == y.view(np.uint64)) | (np.isnan(x) & np.isnan(y))
        if not same.all():
            i = int(np.argmin(same))
            return {"identical": False, "compared": compared,
                    "first": {"node": nid, "origin": o, "index": i, "want": float(x[i]), "got": float(y[i])}}
        compared += 1
    return {"identical": True, "compared": compared, "first": None}


def _ratio(gpu, ref, bound):
    gpu = np.asarray(gpu, dtype=np.float64).reshape(-1)
    d = np.abs(gpu - ref)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = d / (S * bound)
    r = np.where(d == 0, 0.0, r)
    r = np.where(np.isnan(d), np.inf, r)
    r = np.where(np.isnan(r), np.inf, r)
    return r


def judge(graph, gpu, values, bounds, only=None):
    """src/gpu/bounds.js:155-171: pass iff |gpu - ref| <= 2 E everywhere."""
    worst, first = 0.0, None
    for node in graph.nodes:
        if only is not None and node.id not in only:
            continue
        r = _ratio(gpu[node.id], values[node.id], bounds[node.id])
        if r.size:
            w = float(r.max())
            worst = max(worst, w)
            if w > 1 and first is None:
                i = int(np.argmax(r > 1))
                first = {"node": node.id, "op": node.op, "index": i, "gpu": float(np.asarray(gpu[node.id]).reshape(-1)[i]),
                         "ref": float(values[node.id][i]), "bound": float(bounds[node.id][i]), "ratio": float(r[i])}
    return {"pass": first is None, "worst": worst, "first": first}


def unjudgeable(values, bounds):
    """src/gpu/bounds.js:139-148."""
    count = 0
    for v, b in zip(values, bounds):
        if v is None:
            continue
        count += int((~np.isfinite(v) | (np.abs(v) > F32_MAX) | ~np.isfinite(b)).sum())
    return count


def judge_fused(fused, gpu, values, bounds):
    """Every surviving node of a fused graph against the original's reference (harness-m4.js:46-60)."""
    worst, first = 0.0, None
    for node in fused.graph.nodes:
        o = fused.origin[node.id]
        g = np.asarray(gpu[node.id]).reshape(-1)
        if g.size != values[o].size:
            return {"pass": False, "worst": math.inf, "first": {"node": node.id, "origin": o, "reason": "length"}}
        r = _ratio(g, values[o], bounds[o])
        if r.size:
            w = float(r.max())
            worst = max(worst, w)
            if w > 1 and first is None:
                i = int(np.argmax(r > 1))
                first = {"node": node.id, "origin": o, "op": node.op, "pattern": node.attrs.get("pattern"),
                         "index": i, "gpu": float(g[i]), "ref": float(values[o][i]), "bound": float(bounds[o][i]),
                         "ratio": float(r[i])}
    return {"pass": first is None, "worst": worst, "first": first}


def judge_outputs(values, bounds, gpu):
    """Outputs against the reference with the 1% unjudgeable rule (src/fusion/workloads.js:351-367)."""
    worst, first, unj, elements = 0.0, None, 0, 0
    for k, (v, b, g) in enumerate(zip(values, bounds, gpu)):
        g = np.asarray(g, dtype=np.float64).reshape(-1)
        bad = ~np.isfinite(v) | (np.abs(v) > F32_MAX) | ~np.isfinite(b)
        elements += v.size
        unj += int(bad.sum())
        r = np.where(bad, 0.0, _ratio(g, v, b))
        if r.size:
            w = float(r.max())
            worst = max(worst, w)
            if w > 1 and first is None:
                i = int(np.argmax(r > 1))
                first = {"output": k, "index": i, "gpu": float(g[i]), "ref": float(v[i]), "bound": float(b[i]),
                         "ratio": float(r[i])}
    unjudged = unj > 0.01 * elements
    return {"pass": first is None and not unjudged, "unjudged": unjudged, "worst": worst, "unjudgeable": unj,
            "elements": elements, "first": first}


def local_reference_fused(graph, values):
    """Node-local expectations: each launched node on float32-rounded operands (harness-m4.js:182-200)."""
    pkg = _pkg()
    expected = [None] * len(graph.nodes)
    bound = [None] * len(graph.nodes)
    for node in graph.nodes:
        if node.op in ("input", "const"):
            continue
        if node.op == "fused":
            g = pkg.fuse.body_of(node)
            out = node.attrs["output"]
        else:
            g = pkg.ir.Graph()
            ins = [g.input(f"a{k}", graph.nodes[i].shape) for k, i in enumerate(node.inputs)]
            out = g.emit(node.op, ins, node.attrs)
        v, b, _ = reference_with_bounds(g, {f"a{k}": values[i] for k, i in enumerate(node.inputs)}, want=[out])
        expected[node.id] = v[out]
        bound[node.id] = b[out]
    return expected, bound


def tensor_score(ours, ref, rtol=1e-12, atol_scale=1e-12):
    """Metric v2 (src/testing/golden.js:36-49): largest |ours-ref| / (atol + rtol |ref|)."""
    ours = np.asarray(ours, dtype=np.float64).reshape(-1)
    ref = np.asarray(ref, dtype=np.float64).reshape(-1)
    if ours.size != ref.size:
        return math.inf
    if ref.size == 0:
        return 0.0
    atol = atol_scale * max(1.0, float(np.abs(ref).max()))
    d = np.abs(ours - ref)
    r = d / (atol + rtol * np.abs(ref))
    r = np.where(np.isnan(d), np.inf, r)
    return float(r.max())


def judge_local(graph, gpu, expected, bound):
    """Node-local judging with the 1% unjudgeable rule (src/gpu/harness-m4.js:202-223)."""
    worst, first, unj, elements = 0.0, None, 0, 0
    by_kind = {}
    for node in graph.nodes:
        if expected[node.id] is None:
            continue
        r, e = expected[node.id], bound[node.id]
        g = np.asarray(gpu[node.id], dtype=np.float64).reshape(-1)
        kind = node.attrs.get("pattern", "plain") if node.op == "fused" else "plain"
        k = by_kind.setdefault(kind, {"nodes": 0, "worst": 0.0})
        k["nodes"] += 1
        bad = ~np.isfinite(r) | (np.abs(r) > F32_MAX) | ~np.isfinite(e)
        elements += r.size
        unj += int(bad.sum())
        ratio = np.where(bad, 0.0, _ratio(g, r, e))
        if ratio.size:
            w = float(ratio.max())
            worst = max(worst, w)
            k["worst"] = max(k["worst"], w)
            if w > 1 and first is None:
                i = int(np.argmax(ratio > 1))
                first = {"node": node.id, "op": node.op, "pattern": node.attrs.get("pattern"), "index": i,
                         "gpu": float(g[i]), "ref": float(r[i]), "bound": float(e[i]), "ratio": float(ratio[i])}
    unjudged = unj > 0.01 * elements
    return {"pass": first is None and not unjudged, "unjudged": unjudged, "worst": worst, "first": first,
            "unjudgeable": unj, "elements": elements, "byKind": by_kind}
