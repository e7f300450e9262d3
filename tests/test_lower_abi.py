"""The lowering in the C ABI (tc_lower_json) against the Python host's lowering, on the CPU.

A host holding only libtcb200 -- the reference's JavaScript, say -- lowers a graph in the reference's
Graph.toJSON form through tc_lower_json and gets the launch records back from tc_lowered_json.  Those
records must be the Python host's, field for field: every kernel's CUDA source character for character,
its calls (grid, block, shared memory, parameters, tensor maps, error word, second outputs), scratch,
algorithmic bytes and plan details -- over lower() and lowerFused() of the BASELINE workloads, the
reference's 100 direct cases (each value sabotage too), its 146 golden cases, the transformer's step with
transposes folded, column sums fused and readers computed in their producers' pass, and a sample of the differential-fuzz corpus, on both matmul
paths.  The GPU test (tests/test_gpu_lower_abi.py) then runs lowerings made this way.
"""
import ctypes
import importlib
import json
import os

import pytest

from conftest import GOLDEN


def c_lower(lib, graph, **opts):
    h = ctypes.c_void_p()
    st = lib.tc_lower_json(json.dumps(graph.to_json()).encode(), json.dumps(opts).encode(), ctypes.byref(h))
    assert st == 0, lib.tc_last_error().decode()
    n = ctypes.c_uint64()
    assert lib.tc_lowered_json(h, None, 0, ctypes.byref(n)) == 0
    buf = ctypes.create_string_buffer(n.value)
    assert lib.tc_lowered_json(h, buf, n.value, ctypes.byref(n)) == 0
    lib.tc_lowered_free(h)
    return json.loads(buf.value.decode())


def _py_record(lau):
    def norm(v):
        if isinstance(v, tuple):
            return [norm(x) for x in v]
        return v
    calls = []
    for c in lau.calls:
        calls.append({"name": c.name, "grid": list(c.grid), "block": list(c.block), "smem": c.smem,
                      "params": list(c.params), "err_offset": c.err_offset, "out_node": c.out_node,
                      "ptr_params": [list(p) for p in c.ptr_params],
                      "tma": None if c.tma is None else [list(m) for m in c.tma]})
    rec = {"node": lau.node, "op": lau.op, "kind": lau.kind, "pattern": lau.pattern, "inputs": list(lau.inputs),
           "code": lau.code, "scratch_bytes": lau.scratch_bytes, "bytes": lau.bytes, "calls": calls,
           "info": {k: norm(v) for k, v in (lau.info or {}).items()}}
    nodes = getattr(lau, "nodes", None)
    if nodes:
        rec["nodes"] = list(nodes)
    return rec


def _compare(lib, cg, graph, fused=True, **opts):
    if fused:
        py = cg.lower_fused(graph, **opts)
    else:
        py = cg.lower(graph, **{k: v for k, v in opts.items() if k in ("matmul", "sabotage", "fold", "keep")})
    c = c_lower(lib, graph, fused=fused, **{k: (list(v) if k == "keep" else v) for k, v in opts.items()})
    assert c["folded"] == list(py["folded"])
    assert c.get("transposed", []) == [list(p) for p in py.get("transposed", [])]
    assert len(c["launches"]) == len(py["launches"])
    for k, (a, b) in enumerate(zip(py["launches"], c["launches"])):
        want = _py_record(a)
        for key in want:
            assert b.get(key) == want[key], (k, key, want.get("kind"))
    return len(py["launches"])


@pytest.fixture(scope="module")
def mods(pkg):
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    return rt.lib(), cg, wl


def test_baseline_workloads_lower_identically(pkg, mods):
    lib, cg, wl = mods
    n = 0
    for R, C in ((8192, 8192), (257, 1000), (64, 8192)):
        W = wl.c2_graph(R, C)
        f = pkg.fuse.fuse(W["graph"], keep=W["keep"])
        keep = [f.index[k] for k in W["keep"]]
        n += _compare(lib, cg, f.graph)
        n += _compare(lib, cg, f.graph, colfuse=True, keep=keep)
        n += _compare(lib, cg, f.graph, colfuse=True, mofuse=True, keep=keep)
        n += _compare(lib, cg, f.graph, mofuse=True)
        n += _compare(lib, cg, W["graph"], fused=False)
    for M, K, N in (*wl.C3_SHAPES, (256, 4096, 128), (130, 1024, 96), (2432, 128, 2048), (5120, 256, 1024), (64, 16, 8)):
        for act in ("relu", "tanh"):
            W = wl.c3_graph(M, K, N, act)
            f = pkg.fuse.fuse(W["graph"], keep=W["keep"])
            for mm in ("naive", "tiled"):
                n += _compare(lib, cg, f.graph, matmul=mm)
                n += _compare(lib, cg, W["graph"], fused=False, matmul=mm)
    for what in ("softmax", "logsoftmax", "rowsum"):
        for R, C in ((65536, 4096), (300, 4096), (64, 10), (5, 4097)):
            W = wl.c4_graph(R, C, what)
            f = pkg.fuse.fuse(W["graph"], keep=W["keep"])
            n += _compare(lib, cg, f.graph)
            n += _compare(lib, cg, W["graph"], fused=False)
    step = wl.c1_step(64)
    keep = [step["loss"], *step["outputs"].values()]
    f = pkg.fuse.fuse(step["graph"], keep=keep)
    for mm in ("naive", "tiled"):
        n += _compare(lib, cg, f.graph, matmul=mm)
    assert n > 200


def test_transformer_step_lowers_identically(pkg, mods):
    """The C5 gradient program as the trainer lowers it (tiled GEMMs, folded transposes, fused column
    sums) at the benchmark size, and the Adam program."""
    lib, cg, wl = mods
    s = pkg.steps
    for over in ({}, {"d": 64, "L": 2, "H": 4, "ff": 128, "T": 32, "batch": 4}):
        cfg, c = wl.c5_cfg(**over)
        gs = s.build_grad3b(c["V"], c["batch"], cfg)
        k0 = [gs["loss"], *gs["grads"].values()]
        f = pkg.fuse.fuse(gs["graph"], keep=k0)
        keep = [f.index[i] for i in k0]
        assert _compare(lib, cg, f.graph, matmul="tiled", fold=True, keep=keep, colfuse=True) > 100
        assert _compare(lib, cg, f.graph, matmul="tiled", fold=True, keep=keep, colfuse=True, mofuse=True) > 100
        _compare(lib, cg, f.graph, matmul="tiled", fold=True, keep=keep)
        _compare(lib, cg, f.graph, matmul="tiled")
        ad = s.build_adam_graph(c["V"], cfg)
        fa = pkg.fuse.fuse(ad["graph"], keep=list(ad["outputs"].values()))
        _compare(lib, cg, fa.graph, matmul="tiled")


def test_direct_and_golden_cases_lower_identically(pkg, mods):
    lib, cg, _ = mods
    cases = importlib.import_module("tensor-compiler-webgpu_b200.cases").fused_direct_cases()
    for case in cases:
        f = pkg.fuse.fuse(case["graph"])
        mm = case.get("matmul", "naive")
        _compare(lib, cg, f.graph, matmul=mm)
        _compare(lib, cg, case["graph"], fused=False, matmul=mm)
        for sab in ("epilogue-before-bias", "layernorm-tree-short", "softmax-no-max", "fused-bounds-off-by-one"):
            _compare(lib, cg, f.graph, matmul=mm, sabotage=sab)
    with open(os.path.join(GOLDEN, "cases_torch.json")) as fh:
        gcases = json.load(fh)["cases"]
    with open(os.path.join(GOLDEN, "cases_m3_torch.json")) as fh:
        gcases += json.load(fh)["cases"]["cases"]
    for c in gcases:
        g = pkg.ir.Graph.from_json(c["graph"])
        G = pkg.autodiff.grad(g, c["outputs"], [n.id for n in g.inputs()])
        keep = list(c["outputs"]) + list(G.grads)
        f = pkg.fuse.fuse(G.graph, keep=keep)
        fk = [f.index[k] for k in keep]
        for mm in ("naive", "tiled"):
            _compare(lib, cg, f.graph, matmul=mm)
            _compare(lib, cg, f.graph, matmul=mm, colfuse=True, keep=fk)
            _compare(lib, cg, f.graph, matmul=mm, fold=True, keep=fk)
            _compare(lib, cg, f.graph, matmul=mm, fold=True, colfuse=True, mofuse=True, keep=fk)
            _compare(lib, cg, G.graph, fused=False, matmul=mm)


def test_fuzz_corpus_sample_lowers_identically(pkg, mods):
    lib, cg, _ = mods
    corpus = importlib.import_module("tensor-compiler-webgpu_b200.corpus")
    autodiff = importlib.import_module("tensor-compiler-webgpu_b200.autodiff")
    for i in range(1, 2001, 25):
        p = corpus.corpus_program(i, f32=True)
        G = autodiff.grad(p.graph, p.outputs, [n.id for n in p.graph.inputs()])
        for g, keep in ((p.graph, list(p.outputs)), (G.graph, list(p.outputs) + list(G.grads))):
            f = pkg.fuse.fuse(g, keep=keep)
            fk = [f.index[k] for k in keep]
            for mm in ("naive", "tiled"):
                _compare(lib, cg, f.graph, matmul=mm)
                _compare(lib, cg, f.graph, matmul=mm, colfuse=True, mofuse=True, keep=fk)
                _compare(lib, cg, g, fused=False, matmul=mm)


def test_bad_input_is_an_error_not_a_crash(pkg, mods):
    lib, _, _ = mods
    h = ctypes.c_void_p()
    assert lib.tc_lower_json(b'{"nodes": [{"op": "add", "inputs": [3, 4], "attrs": {}, "shape": [2]}]}', None,
                             ctypes.byref(h)) == 1
    assert b"earlier node" in lib.tc_last_error()
    assert lib.tc_lower_json(b"{not json", None, ctypes.byref(h)) == 1
    assert lib.tc_lower_json(b'{"nodes": []}', b'{"matmul": "fast"}', ctypes.byref(h)) == 1
