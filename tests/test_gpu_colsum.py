"""Column and row sums fused into their elementwise producers, on the B200.

A resident program lowered with `colfuse` runs each sum over axis 0 of an elementwise value inside the
producer's launch (tcb/colsum.cuh).  It keeps the plain column sum's split and per-chunk order, so every
output must be bitwise the same as with the separate launches -- for operands read only by the sum
(never stored), for kept or shared operands (stored and summed in one pass), with one chunk (the sums
written directly) and with many (partials combined by the fixed-order finish) -- and within 2E of the
float64 oracle.  Sums over the last axis of enough rows run the same way (tcb/rowsum.cuh), in the
plain row sum's order.  The data-parallel trainer, which fuses its bias gradients and its layer-norm
row sums so, must give the same loss and parameters as without, bit for bit.
"""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _mods():
    return (importlib.import_module("tensor-compiler-webgpu_b200.runtime"),
            importlib.import_module("tensor-compiler-webgpu_b200.codegen"),
            importlib.import_module("tensor-compiler-webgpu_b200.workloads"))


def _shared(pkg, R, C):
    g = pkg.ir.Graph()
    x = g.input("x", [R, C])
    w = g.input("w", [C])
    y = g.tanh(g.mul(x, w))
    s = g.sum(y, 0, True)
    z = g.exp(g.neg(y))
    rng = np.random.default_rng(R * 7 + C)
    inputs = {"x": rng.standard_normal(R * C).astype(np.float32), "w": rng.standard_normal(C).astype(np.float32)}
    return g, [s, z, y], inputs


def _run(rt, runner, fgraph, lowered, outs, inputs):
    prog = rt.Program(runner, fgraph, lowered, keep=outs)
    try:
        for n in fgraph.inputs():
            prog.write(n.id, inputs[n.attrs["name"]])
        prog.run()
        prog.check_errors()
        return [prog.read(o) for o in outs]
    finally:
        prog.free()


def _rows(pkg, shape, stored):
    g = pkg.ir.Graph()
    C = shape[-1]
    x = g.input("x", list(shape))
    w = g.input("w", [C])
    y = g.tanh(g.mul(x, g.broadcast(w, list(shape))))
    s = g.sum(y, len(shape) - 1, True)
    outs = [s]
    if stored:
        outs.append(g.exp(g.neg(y)))
    rng = np.random.default_rng(int(np.prod(shape)) + C)
    inputs = {"x": rng.standard_normal(int(np.prod(shape))).astype(np.float32),
              "w": rng.standard_normal(C).astype(np.float32)}
    return g, outs, inputs


@pytest.mark.parametrize("case", ["2000x256-stored", "2000x256-sum", "1500x65-stored", "1500x65-sum",
                                  "3x700x64-stored", "4096x1000-sum"])
def test_rowsum_fusion_is_bitwise_the_separate_launches(pkg, oracle, runner, case):
    rt, cg, wl = _mods()
    dims, mode = case.split("-")
    shape = [int(v) for v in dims.split("x")]
    graph, keep, inputs = _rows(pkg, shape, mode == "stored")
    f = pkg.fuse.fuse(graph, keep=keep)
    outs = [f.index[k] for k in dict.fromkeys(keep)]
    plain = cg.lower_fused(f.graph)
    fused = cg.lower_fused(f.graph, colfuse=True, keep=outs)
    rs = [l for l in fused["launches"] if l.kind == "fused-rowsum"]
    assert len(rs) == 1 and rs[0].info["write"] == (mode == "stored")
    a = _run(rt, runner, f.graph, plain, outs, inputs)
    b = _run(rt, runner, f.graph, fused, outs, inputs)
    for o, x, y in zip(outs, a, b):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32)), o
    ks = list(dict.fromkeys(keep))
    values, bounds, _ = oracle.reference_with_bounds(graph, inputs, want=ks)
    j = oracle.judge_outputs([values[k] for k in ks], [bounds[k] for k in ks], b)
    assert j["pass"], j


@pytest.mark.parametrize("case", ["c2-257x1000", "c2-64x8192", "c2-40x300", "shared-300x64", "shared-40x256",
                                  "shared-5000x65"])
def test_colsum_fusion_is_bitwise_the_separate_launches(pkg, oracle, runner, case):
    rt, cg, wl = _mods()
    kind, dims = case.split("-")
    R, C = map(int, dims.split("x"))
    if kind == "c2":
        W = wl.c2_graph(R, C)
        graph, keep, inputs = W["graph"], W["keep"], wl.c2_inputs(W)
    else:
        graph, keep, inputs = _shared(pkg, R, C)
    f = pkg.fuse.fuse(graph, keep=keep)
    outs = [f.index[k] for k in dict.fromkeys(keep)]
    plain = cg.lower_fused(f.graph)
    fused = cg.lower_fused(f.graph, colfuse=True, keep=outs)
    assert any(l.kind == "fused-colsum" for l in fused["launches"])
    a = _run(rt, runner, f.graph, plain, outs, inputs)
    b = _run(rt, runner, f.graph, fused, outs, inputs)
    for o, x, y in zip(outs, a, b):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32)), o
    values, bounds, _ = oracle.reference_with_bounds(graph, inputs, want=list(dict.fromkeys(keep)))
    ks = list(dict.fromkeys(keep))
    j = oracle.judge_outputs([values[k] for k in ks], [bounds[k] for k in ks], b)
    assert j["pass"], j


@pytest.mark.parametrize("rows", [128, 2048])
def test_dp_trainer_with_fused_bias_gradients_is_bitwise_unchanged(pkg, runner, rows):
    """128 token rows: column sums only; 2048: the layer-norm and attention row sums fused as well."""
    rt, cg, wl = _mods()
    dp = importlib.import_module("tensor-compiler-webgpu_b200.dp")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=64, L=2, H=4, ff=128, T=32 if rows == 128 else 64, batch=rows // (32 if rows == 128 else 64))
    V, B = c["V"], c["batch"]
    params = s.init_params_normal(V, 0, 0.02, cfg)
    a = dp.DPTrainer(runner, V, B, cfg, params, colfuse=False)
    b = dp.DPTrainer(runner, V, B, cfg, params, colfuse=True)
    try:
        assert sum(1 for l in b.grad_prog.launches if l.kind == "fused-colsum") >= 10
        assert (sum(1 for l in b.grad_prog.launches if l.kind == "fused-rowsum") >= 10) == (rows == 2048)
        assert b.grad_prog.kernel_launches < a.grad_prog.kernel_launches
        for t in range(3):
            x, y = wl.one_hot_batch(wl.c5_tokens(B, cfg["T"], V, seed=t), V)
            la, lb = a.train(x, y), b.train(x, y)
            assert np.float32(la).tobytes() == np.float32(lb).tobytes(), t
        pa, pb = a.read(a.names), b.read(b.names)
        for n in a.names:
            assert np.array_equal(pa[n].view(np.uint32), pb[n].view(np.uint32)), n
    finally:
        a.destroy()
        b.destroy()
