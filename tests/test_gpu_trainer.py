"""The persistent training step on the B200.

* The fused trainer (one native plan, replayed as a CUDA graph, parameters and
  state fed back on the device) against the checked path -- the same fused
  launches run one by one through GpuRunner.run with the feedback done on the
  host -- bit for bit (src/gpu/harness-m4.js:310-330, runConsistencyM4).
* The data-parallel trainer at world size 1 (gradient graph, Adam graph)
  against the single fused step graph: the same mathematics partitioned
  differently, so within float32 tolerance rather than bitwise.
"""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_fused_trainer_matches_checked_path_bitwise(pkg, runner):
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    s = pkg.steps
    step = s.build_mlp_step(wl.C1_DIMS, 64, opt=s.ADAM, hidden="tanh")
    fstep = rt.fused_step(step)
    data = wl.c1_inputs(64)
    params = {k: data[k] for k in s.PARAMS}
    state = s.mlp_initial_state(s.ADAM, wl.C1_DIMS)
    tr = rt.FusedTrainer(runner, fstep, params, state)
    cur = {**{k: np.asarray(v, np.float32) for k, v in params.items()},
           **{k: np.asarray(v, np.float32) for k, v in state.items()}}
    names = list(params) + list(state)
    try:
        for it in range(3):
            x = data["x"] if it % 2 == 0 else data["x"][::-1].copy()
            loss = tr.train(x, data["y"])
            feed = {**cur, "x": x, "y": data["y"], step["cotangent"]: [1.0]}
            g = fstep["graph"]
            out = runner.run(g, fstep["lowered"], {n.attrs["name"]: feed[n.attrs["name"]] for n in g.inputs()})
            assert np.float32(loss).tobytes() == out["values"][fstep["loss"]].tobytes(), it
            cur = {k: out["values"][fstep["outputs"][k]] for k in names}
        got = tr.read(names)
        for k in names:
            assert np.array_equal(got[k].view(np.uint32), cur[k].view(np.uint32)), k
    finally:
        tr.destroy()


@pytest.mark.parametrize("split_mode,rtol,atol", [("0", 1e-4, 1e-6), (None, 1e-3, 1e-5)])
def test_dp_trainer_world1_matches_fused_step(pkg, runner, monkeypatch, split_mode, rtol, atol):
    """The data-parallel trainer at world size 1 against the fused step.  With every GEMM operand split
    by a split pass ("0") both compute the same products; by default the folded program may split an
    operand inside the GEMM where the unfolded one cannot (hi = trunc(x) there, rna(x) in the pass), so
    the parameters after three Adam steps agree to the looser tolerance."""
    if split_mode is not None:
        monkeypatch.setenv("TCB_GEMM_FUSED", split_mode)
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    dp = importlib.import_module("tensor-compiler-webgpu_b200.dp")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=64, L=2, H=4, ff=128, T=32, batch=4)
    V, B = c["V"], c["batch"]
    params = s.init_params_normal(V, 0, 0.02, cfg)
    state = s.adam_initial_state(s.param_names(V, cfg), s.param_shapes(V, cfg))
    x, y = wl.one_hot_batch(wl.c5_tokens(B, cfg["T"], V), V)
    one = rt.fused_step(s.build_step3b(V, B, cfg), matmul="tiled")
    ref = rt.FusedTrainer(runner, one, params, state)
    tr = dp.DPTrainer(runner, V, B, cfg, params, matmul="tiled")
    try:
        for it in range(3):
            la = ref.train(x, y)
            lb = tr.train(x, y)
            assert abs(la - lb) <= 1e-5 * max(1.0, abs(la)), (it, la, lb)
        pa = ref.read(tr.names)
        pb = tr.read(tr.names)
        for k in tr.names:
            np.testing.assert_allclose(pb[k], pa[k], rtol=rtol, atol=atol, err_msg=k)
    finally:
        ref.destroy()
        tr.destroy()


def test_folded_transposes_and_aliased_reshapes_change_no_bit(pkg, runner, monkeypatch):
    """The resident program (transposes folded into GEMM operand splits, reshapes aliased) gives the
    verification path's values bit for bit on the loss and every gradient, with every GEMM operand
    split by a split pass.  (A fold can change whether an operand qualifies for the in-kernel split --
    its raw row stride is K or M -- and that split takes hi = trunc(x) instead of rna(x): same budget,
    other bits.)"""
    monkeypatch.setenv("TCB_GEMM_FUSED", "0")
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=64, L=2, H=4, ff=128, T=32, batch=4)
    V, B = c["V"], c["batch"]
    gs = s.build_grad3b(V, B, cfg)
    f = pkg.fuse.fuse(gs["graph"], keep=[gs["loss"], *gs["grads"].values()])
    keep = [f.index[i] for i in [gs["loss"], *gs["grads"].values()]]
    params = s.init_params_normal(V, 0, 0.02, cfg)
    x, y = wl.one_hot_batch(wl.c5_tokens(B, cfg["T"], V), V)
    feed = {**params, "x": x, "y": y, gs["cotangent"]: [1.0]}
    plain = runner.run(f.graph, cg.lower_fused(f.graph, matmul="tiled"),
                       {n.attrs["name"]: feed[n.attrs["name"]] for n in f.graph.inputs()})
    low = cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep)
    assert low["folded"], "the C5 backward has transposes feeding GEMMs"
    prog = rt.Program(runner, f.graph, low, keep=keep)
    try:
        assert prog.alias, "the C5 graph has plain reshapes to alias"
        for n in f.graph.inputs():
            prog.write(n.id, feed[n.attrs["name"]])
        prog.run()
        prog.check_errors()
        for k in keep:
            assert np.array_equal(prog.read(k).view(np.uint32), plain["values"][k].view(np.uint32)), k
    finally:
        prog.free()


def test_streamed_program_matches_step_by_step(pkg, runner):
    """Pipelined steps (copies overlapped across steps, two device slots) give each step's own results."""
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    W = wl.c2_graph(256, 1024)
    f = pkg.fuse.fuse(W["graph"], keep=W["keep"])
    low = cg.lower_fused(f.graph)
    outs = [f.index[k] for k in W["keep"]]
    ins = [n.id for n in f.graph.inputs()]
    sp = rt.StreamedProgram(runner, f.graph, low, ins, outs, slots=2)
    steps, hosts, want = 5, [], []
    try:
        for s in range(steps):
            data = wl.c2_inputs(W, seed=s + 1)
            hin = {n.id: rt.PinnedHost(data[n.attrs["name"]].nbytes) for n in f.graph.inputs()}
            for n in f.graph.inputs():
                hin[n.id].array(data[n.attrs["name"]].size)[:] = data[n.attrs["name"]]
            hout = {o: rt.PinnedHost(pkg.ir.size(f.graph.nodes[o].shape) * 4) for o in outs}
            hosts.append((hin, hout))
            ref = runner.run(f.graph, low, {n.attrs["name"]: data[n.attrs["name"]] for n in f.graph.inputs()})
            want.append({o: ref["values"][o] for o in outs})
        for hin, hout in hosts:
            sp.submit({k: (h.ptr, h.nbytes) for k, h in hin.items()}, {k: (h.ptr, h.nbytes) for k, h in hout.items()})
        sp.drain()
        for s, (hin, hout) in enumerate(hosts):
            for o in outs:
                got = hout[o].array(hout[o].nbytes // 4)
                assert np.array_equal(got.view(np.uint32), want[s][o].view(np.uint32)), (s, o)
    finally:
        sp.free()
        for hin, hout in hosts:
            for h in list(hin.values()) + list(hout.values()):
                h.free()


def test_batched_program_changes_no_bit(pkg, runner):
    """The data-parallel trainer with its resident programs batched (small same-source launches as one
    multi-instance launch, the weight operand splits hoisted into one launch, the feedback copies as
    one launch) against the same trainer unbatched: bit for bit, and with fewer launches."""
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    dp = importlib.import_module("tensor-compiler-webgpu_b200.dp")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=64, L=2, H=4, ff=128, T=32, batch=4)
    V, B = c["V"], c["batch"]
    params = s.init_params_normal(V, 0, 0.02, cfg)
    x, y = wl.one_hot_batch(wl.c5_tokens(B, cfg["T"], V), V)
    a = dp.DPTrainer(runner, V, B, cfg, params, batch=False)
    b = dp.DPTrainer(runner, V, B, cfg, params, batch=True)
    try:
        assert b.kernel_launches < a.kernel_launches
        assert b.grad_prog.hoisted and any(isinstance(l, pkg_runtime().MultiLaunch) for l in b.adam_prog.launches)
        for _ in range(2):
            la, lb = a.train(x, y), b.train(x, y)
            assert np.float32(la).view(np.uint32) == np.float32(lb).view(np.uint32)
        pa, pb = a.read(a.names), b.read(b.names)
        for k in a.names:
            assert np.array_equal(pa[k].view(np.uint32), pb[k].view(np.uint32)), k
    finally:
        a.destroy()
        b.destroy()


def pkg_runtime():
    return importlib.import_module("tensor-compiler-webgpu_b200.runtime")
