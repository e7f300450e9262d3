"""The BASELINE workloads on the B200 against the float64 oracle, at sizes the oracle finishes in seconds,
plus size-independent properties at the full sizes."""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def wl():
    return importlib.import_module("tensor-compiler-webgpu_b200.workloads")


@pytest.fixture(scope="module")
def cg():
    return importlib.import_module("tensor-compiler-webgpu_b200.codegen")


def _judge_run(pkg, oracle, runner, cg, graph, inputs, keep, matmul="naive"):
    values, bounds, rounded = oracle.reference_with_bounds(graph, inputs)
    fused = pkg.fuse.fuse(graph, keep=keep)
    gf = runner.run(fused.graph, cg.lower_fused(fused.graph, matmul=matmul), rounded, canary=True)
    assert all(gf["canaryIntact"])
    outs = [fused.index[k] for k in keep]
    j = oracle.judge_outputs([values[k] for k in keep], [bounds[k] for k in keep], [gf["values"][o] for o in outs])
    return j, fused, gf


def test_c1_mlp_forward_backward(pkg, oracle, runner, wl, cg):
    step = wl.c1_step(64)
    inputs = wl.c1_inputs(64)
    inputs[step["cotangent"]] = [1.0]
    keep = [step["loss"], *step["outputs"].values()]
    j, _, _ = _judge_run(pkg, oracle, runner, cg, step["graph"], inputs, keep)
    assert j["pass"], j


@pytest.mark.parametrize("R,C", [(64, 8192), (257, 1000)])
def test_c2_chain_forward_backward(pkg, oracle, runner, wl, cg, R, C):
    W = wl.c2_graph(R, C)
    inputs = wl.c2_inputs(W)
    j, _, _ = _judge_run(pkg, oracle, runner, cg, W["graph"], inputs, W["keep"])
    assert j["pass"], j


@pytest.mark.parametrize("what", ["softmax", "logsoftmax", "rowsum"])
@pytest.mark.parametrize("R,C", [(300, 4096), (64, 10), (5, 4097)])
def test_c4_rowwise_forward_backward(pkg, oracle, runner, wl, cg, what, R, C):
    W = wl.c4_graph(R, C, what)
    inputs, hot = wl.c4_inputs(W)
    j, fused, gf = _judge_run(pkg, oracle, runner, cg, W["graph"], inputs, W["keep"])
    assert j["pass"], j
    if what == "softmax":  # rows offset by +800 stay finite and sum to 1
        y = gf["values"][fused.index[W["output"]]].reshape(R, C)
        assert np.isfinite(y).all()
        assert np.allclose(y.sum(axis=1), 1.0, atol=1e-4)


@pytest.mark.parametrize("M,K,N", [(256, 4096, 128), (130, 1024, 96)])
@pytest.mark.parametrize("act", ["relu", "tanh"])
def test_c3_matmul_epilogue(pkg, oracle, runner, wl, cg, M, K, N, act):
    W = wl.c3_graph(M, K, N, act)
    inputs = wl.c3_inputs(M, K, N)
    for matmul in ("naive", "tiled"):
        j, fused, _ = _judge_run(pkg, oracle, runner, cg, W["graph"], inputs, W["keep"], matmul=matmul)
        assert [n.attrs["kind"] for n in fused.graph.nodes if n.op == "fused"] == ["epilogue"]
        assert j["pass"], (matmul, j)


@pytest.mark.parametrize("M,K,N,tail", [(3456, 512, 2048, 2), (5760, 512, 1024, 4)])
def test_c3_last_wave_split(pkg, oracle, runner, wl, cg, M, K, N, tail):
    """Shapes whose last wave of output tiles is cut into K ranges (reduced by the last arriver):
    judged against the oracle, and bitwise the same on a second run."""
    W = wl.c3_graph(M, K, N, "tanh")
    inputs = wl.c3_inputs(M, K, N)
    fused = pkg.fuse.fuse(W["graph"], keep=W["keep"])
    lowered = cg.lower_fused(fused.graph, matmul="tiled")
    assert [l.info["tail_split"] for l in lowered["launches"] if l.info.get("path") == "tcgen05-3xtf32"] == [tail]
    j, fused, gf = _judge_run(pkg, oracle, runner, cg, W["graph"], inputs, W["keep"], matmul="tiled")
    assert j["pass"], j
    o = fused.index[W["keep"][0]]
    rounded = {k: np.asarray(v, np.float32).astype(np.float64) for k, v in inputs.items()}
    again = runner.run(fused.graph, cg.lower_fused(fused.graph, matmul="tiled"), rounded)
    assert np.array_equal(gf["values"][o], again["values"][o])


def test_transformer_step_node_local(pkg, oracle, runner, wl, cg):
    """A C5-shaped training step (forward + backward + Adam) at reduced sizes, judged node by node.

    The reference judges its fused training step this way (src/gpu/harness-m4.js:225-268): every launch
    runs on float32-rounded reference operands and is held to its own body's composed budget.
    """
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    cfg, c = wl.c5_cfg(d=32, L=1, H=2, ff=64, T=16, batch=2)
    V = c["V"]
    s = pkg.steps
    st = s.build_step3b(V, c["batch"], cfg)
    params = s.init_params_normal(V, 0, 0.02, cfg)
    state = s.adam_initial_state(st["names"], s.param_shapes(V, cfg))
    x, y = wl.one_hot_batch(wl.c5_tokens(c["batch"], cfg["T"], V), V)
    inputs = {**params, **state, "x": x, "y": y, st["cotangent"]: [1.0]}
    keep = [st["loss"], st["logits"], *st["outputs"].values()]
    values, _, _ = oracle.reference_with_bounds(st["graph"], inputs)
    fused = pkg.fuse.fuse(st["graph"], keep=keep)
    fvals = [values[o] for o in fused.origin]
    expected, bound = oracle.local_reference_fused(fused.graph, fvals)
    lowered = cg.lower_fused(fused.graph)
    gpu = rt.run_local(runner, fused.graph, lowered, fvals, canary=True)
    j = oracle.judge_local(fused.graph, gpu, expected, bound)
    assert j["pass"], {k: v for k, v in j.items() if k != "byKind"}
    assert {"matmul-epilogue", "elementwise"} <= set(j["byKind"])


@pytest.mark.parametrize("a_t,b_t", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("mode,fs", [("1", (True, True)), ("0", (False, False)), ("a", (True, False)),
                                     ("b", (False, True))])
def test_gemm_operand_layouts(pkg, oracle, runner, wl, cg, monkeypatch, a_t, b_t, mode, fs):
    """Both operands K-major or MN-major (a folded transposeLast2 reads the transpose's source), each
    split inside the GEMM or by a split pass: judged against the oracle."""
    monkeypatch.setenv("TCB_GEMM_FUSED", mode)
    from importlib import import_module
    ir = import_module("tensor-compiler-webgpu_b200.ir")
    Bt, M, K, N = 3, 200, 96, 136
    g = ir.Graph()
    x = g.input("x", [Bt, K, M] if a_t else [Bt, M, K])
    y = g.input("y", [Bt, N, K] if b_t else [Bt, K, N])
    bias = g.input("bias", [N])
    a = g.transpose(x, [0, 2, 1]) if a_t else x
    b = g.transpose(y, [0, 2, 1]) if b_t else y
    out = g.tanh(g.add(g.matmul(a, b), bias))
    rng = pkg.rng.Rng(7)
    inputs = {"x": rng.normal_array(Bt * M * K, 0, K ** -0.5).astype(np.float32),
              "y": rng.normal_array(Bt * K * N, 0, K ** -0.5).astype(np.float32),
              "bias": rng.normal_array(N, 0, 0.3).astype(np.float32)}
    values, bounds, rounded = oracle.reference_with_bounds(g, inputs)
    fused = pkg.fuse.fuse(g, keep=[out])
    o = fused.index[out]
    lowered = cg.lower_fused(fused.graph, matmul="tiled", fold=True, keep=[o])
    tc = [l for l in lowered["launches"] if l.info and l.info.get("path") == "tcgen05-3xtf32"]
    assert [(l.info["a_t"], l.info["b_t"], l.info["fused_split"]) for l in tc] == [(a_t, b_t, fs)]
    prog = pkg_runtime().Program(runner, fused.graph, lowered, keep=[o])
    try:
        for n in fused.graph.inputs():
            prog.write(n.id, rounded[n.attrs["name"]].astype(np.float32))
        prog.run()
        runner.sync()
        prog.check_errors()
        got = prog.read(o)
    finally:
        prog.free()
    j = oracle.judge_outputs([values[out]], [bounds[out]], [got])
    assert j["pass"], j


@pytest.mark.parametrize("a_t,b_t", [(False, False), (True, True)])
def test_gemm_last_wave_split_with_in_kernel_operand_split(pkg, oracle, runner, cg, a_t, b_t):
    """150 batched 128 x 1024 x 64 products: 150 tiles on 148 CTAs, so the last two tiles are cut into K
    ranges (K has 32 K-blocks: long enough to split), while both operands are split inside the GEMM
    (each is loaded by one tile): judged against the oracle."""
    from importlib import import_module
    ir = import_module("tensor-compiler-webgpu_b200.ir")
    Bt, M, K, N = 150, 128, 1024, 64
    g = ir.Graph()
    x = g.input("x", [Bt, K, M] if a_t else [Bt, M, K])
    y = g.input("y", [Bt, N, K] if b_t else [Bt, K, N])
    a = g.transpose(x, [0, 2, 1]) if a_t else x
    b = g.transpose(y, [0, 2, 1]) if b_t else y
    out = g.relu(g.matmul(a, b))
    rng = pkg.rng.Rng(11)
    inputs = {"x": rng.normal_array(Bt * M * K, 0, K ** -0.5).astype(np.float32),
              "y": rng.normal_array(Bt * K * N, 0, K ** -0.5).astype(np.float32)}
    values, bounds, rounded = oracle.reference_with_bounds(g, inputs)
    fused = pkg.fuse.fuse(g, keep=[out])
    o = fused.index[out]
    lowered = cg.lower_fused(fused.graph, matmul="tiled", fold=True, keep=[o])
    tc = [l for l in lowered["launches"] if l.info and l.info.get("path") == "tcgen05-3xtf32"]
    assert [(l.info["tail_split"] > 1, l.info["fused_split"]) for l in tc] == [(True, (True, True))]
    prog = pkg_runtime().Program(runner, fused.graph, lowered, keep=[o])
    try:
        for n in fused.graph.inputs():
            prog.write(n.id, rounded[n.attrs["name"]].astype(np.float32))
        prog.run()
        runner.sync()
        prog.check_errors()
        got = prog.read(o)
    finally:
        prog.free()
    j = oracle.judge_outputs([values[out]], [bounds[out]], [got])
    assert j["pass"], j


def pkg_runtime():
    return importlib.import_module("tensor-compiler-webgpu_b200.runtime")
