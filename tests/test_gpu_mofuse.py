"""Elementwise readers computed in their producer's pass, on the B200.

A resident program lowered with `mofuse` computes an elementwise reader inside its elementwise
producer's launch (tcb/elementwise_mo.cuh) and stores both.  Each output takes the same operations as
in its own launch, so every output must be bitwise that of the separate launches -- the C2 chain at
two sizes (together with the fused column sum), a producer with a broadcast reader -- and within 2E
of the float64 oracle; the data-parallel trainer, which lowers its gradient program so, must give the
same loss and parameters as without it, bit for bit, over three steps.
"""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _mods():
    return (importlib.import_module("tensor-compiler-webgpu_b200.runtime"),
            importlib.import_module("tensor-compiler-webgpu_b200.codegen"),
            importlib.import_module("tensor-compiler-webgpu_b200.workloads"))


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


def _reader_graph(pkg, R, C):
    g = pkg.ir.Graph()
    x = g.input("x", [R, C])
    p = g.exp(g.mul(x, g.input("w", [R, C])))
    q = g.div(p, g.broadcast(g.input("row", [C]), [R, C]))
    r = g.tanh(p)
    rng = np.random.default_rng(R + C)
    ins = {"x": (rng.standard_normal(R * C) * 0.5).astype(np.float32),
           "w": rng.standard_normal(R * C).astype(np.float32),
           "row": rng.uniform(0.5, 2.0, C).astype(np.float32)}
    return g, [p, q, r], ins


@pytest.mark.parametrize("case", ["c2-257x1000", "c2-64x8192", "reader-300x256"])
def test_multi_output_launches_are_bitwise_the_separate_ones(pkg, oracle, runner, case):
    rt, cg, wl = _mods()
    kind, dims = case.split("-")
    R, C = map(int, dims.split("x"))
    if kind == "c2":
        W = wl.c2_graph(R, C)
        graph, keep, inputs = W["graph"], W["keep"], wl.c2_inputs(W)
    else:
        graph, keep, inputs = _reader_graph(pkg, R, C)
    f = pkg.fuse.fuse(graph, keep=keep)
    outs = [f.index[k] for k in dict.fromkeys(keep)]
    plain = cg.lower_fused(f.graph)
    fused = cg.lower_fused(f.graph, colfuse=True, mofuse=True, keep=outs)
    assert any(l.kind == "fused-multi" for l in fused["launches"])
    a = _run(rt, runner, f.graph, plain, outs, inputs)
    b = _run(rt, runner, f.graph, fused, outs, inputs)
    for o, x, y in zip(outs, a, b):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32)), o
    ks = list(dict.fromkeys(keep))
    values, bounds, _ = oracle.reference_with_bounds(graph, inputs, want=ks)
    j = oracle.judge_outputs([values[k] for k in ks], [bounds[k] for k in ks], b)
    assert j["pass"], j


def test_dp_trainer_with_multi_output_launches_is_bitwise_unchanged(pkg, runner):
    rt, cg, wl = _mods()
    dp = importlib.import_module("tensor-compiler-webgpu_b200.dp")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=64, L=2, H=4, ff=128, T=32, batch=4)
    V, B = c["V"], c["batch"]
    params = s.init_params_normal(V, 0, 0.02, cfg)
    a = dp.DPTrainer(runner, V, B, cfg, params, mofuse=False)
    b = dp.DPTrainer(runner, V, B, cfg, params, mofuse=True)
    try:
        assert sum(1 for l in b.grad_prog.launches if l.kind == "fused-multi") >= 10
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
