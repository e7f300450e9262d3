"""The resident trainers on the B200 judged against the float64 oracle.

The trainers are the product's training path: one resident Program per graph (lifetime-planned arena,
aliased reshapes, batched small launches, hoisted weight splits, the native plan replayed as one CUDA
graph) with parameters and optimizer state fed back on the device.

* MLP, free-running (src/gpu/harness-m3.js:107-137, runFreeRunning): the reference's own 8 runs of
  golden/train-spec-m3.json (SGD and Adam, 8 -> 16 -> 4 relu, batch 32) on FusedTrainer, 5 steps each.
  The trainer continues from its own parameters and state, the oracle from its float64 values, and each
  step's reference carries the previous step's values with their bounds (bounds.js's `carried` form,
  src/gpu/bounds.js:86-102).  The loss and every updated parameter and state tensor must lie within 2E.
  As in the reference, a run stops at the first step whose reference has an unjudgeable element
  (harness-m3.js:45: the budget is first order and Adam's normalisation outgrows it after a few steps;
  the reference's own record skips 3 of its 8 runs early).
* Decoder transformer (the C5 model family): its composed end-to-end bound is too loose to judge a whole
  step, so -- as the reference judges its transformer step, node-locally (harness-m4.js:182-268) -- the
  resident gradient program of DPTrainer (world size 1, transposes folded into GEMM operands, weight splits
  hoisted, small launches batched) and of FusedTrainer runs with every value kept, each launch is judged
  against the float64 evaluation of its own body on the GPU's float32 operands, and the trainer's arena
  program must reproduce that keep-everything program's loss and gradients bit for bit (an arena reuse
  bug would change them).  The Adam program is judged end to end from the GPU's gradients.  3 steps, each
  from the parameters the trainer itself produced.
"""
import importlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _mods():
    return (importlib.import_module("tensor-compiler-webgpu_b200.runtime"),
            importlib.import_module("tensor-compiler-webgpu_b200.workloads"),
            importlib.import_module("tensor-compiler-webgpu_b200.dp"),
            importlib.import_module("tensor-compiler-webgpu_b200.codegen"))


# ---------------------------------------------------------------- MLP, free-running with carried bounds
def _gather(data, idx, features, classes):
    """src/train/data.js:76-83."""
    x = np.asarray(data["x"], np.float64).reshape(-1, features)[idx].reshape(-1)
    y = np.zeros((len(idx), classes))
    y[np.arange(len(idx)), np.asarray(data["y"])[idx]] = 1
    return x.astype(np.float32), y.reshape(-1).astype(np.float32)


def test_fused_trainer_mlp_free_running_reference_runs(pkg, oracle, runner):
    rt, wl, _, _ = _mods()
    s = pkg.steps
    with open(os.path.join(GOLDEN, "train_m3.json")) as f:
        spec = json.load(f)
    dims = spec["dims"]
    judged = {}
    for cfg in spec["configs"]:
        step = s.build_mlp_step(dims, cfg["batch"], opt=cfg["optimizer"])
        params = {p: np.asarray(cfg["init"][p], np.float32) for p in s.PARAMS}
        state = s.mlp_initial_state(cfg["optimizer"], dims)
        names = list(params) + list(state)
        tr = rt.FusedTrainer(runner, rt.fused_step(step), params, state)
        batches = [_gather(spec["synthetic"]["train"], cfg["schedule"][t], dims["inputs"], dims["classes"])
                   for t in range(5)]

        def gpu_step(xb, yb, tr=tr, names=names):
            return tr.train(xb, yb), tr.read(names)
        try:
            # step 0's reference takes the recorded float32 initial values (no carried bounds yet)
            first = {**params, **{k: np.asarray(v, np.float32) for k, v in state.items()}}
            carried, cur, worsts = None, first, []
            for t, (x, y) in enumerate(batches):
                feed = {**cur, "x": x, "y": y, step["cotangent"]: [1.0]}
                values, bounds, _ = oracle.reference_with_bounds(step["graph"], feed, carried=carried)
                loss, got = gpu_step(x, y)
                if oracle.unjudgeable(values, bounds) > 0:
                    break
                outs = [step["outputs"][n] for n in names]
                j = oracle.judge_outputs([values[step["loss"]]] + [values[o] for o in outs],
                                         [bounds[step["loss"]]] + [bounds[o] for o in outs],
                                         [np.float32([loss])] + [got[n] for n in names])
                assert j["pass"], (cfg["name"], t, j)
                worsts.append(j["worst"])
                carried = {n: (values[step["outputs"][n]], bounds[step["outputs"][n]]) for n in names}
                cur = {n: got[n] for n in names}
        finally:
            tr.destroy()
        judged[cfg["name"]] = worsts
    assert all(len(w) >= 1 for w in judged.values()), judged
    assert all(len(w) == 5 for n, w in judged.items() if n.startswith("sgd")), judged
    assert sum(len(w) for w in judged.values()) >= 26, judged


# ---------------------------------------------------------------- transformer, node-local on resident programs
def _small_transformer(wl):
    cfg, c = wl.c5_cfg(d=64, L=2, H=4, ff=128, T=32, batch=4)
    return cfg, c["V"], c["batch"]


def _keep_all(rt, runner, graph, lowered):
    gone = set(lowered["folded"]) | {m for _, m in lowered.get("transposed", [])}
    ids = [n.id for n in graph.nodes if n.op not in ("input", "const") and n.id not in gone]
    return rt.Program(runner, graph, lowered, keep=ids, batch=True), ids


def _node_local(pkg, oracle, graph, lowered, feed, got):
    """Judge every launched node of `graph` on its own operands (harness-m4.js:182-223); `got` holds the
    GPU value of every launched node, `feed` the inputs' float32 values."""
    vals = [None] * len(graph.nodes)
    folded = set(lowered["folded"])
    # a matmul computed as its reader's transposed product has no launch of its own: its value is that
    # transpose's GPU value transposed back (no arithmetic), and the matmul is judged on it
    tmat = {m: t for t, m in lowered.get("transposed", [])}
    for n in graph.nodes:
        if n.op == "input":
            vals[n.id] = np.asarray(feed[n.attrs["name"]], np.float32).reshape(-1).astype(np.float64)
        elif n.op == "const":
            v = n.attrs["value"]
            vals[n.id] = (np.full(max(1, pkg.ir.size(n.shape)), v, np.float32) if isinstance(v, (int, float))
                          else np.asarray(v, np.float32)).reshape(-1)[:pkg.ir.size(n.shape)].astype(np.float64)
        elif n.id in folded:   # no launch: the transpose of its source, moved on the host (no arithmetic)
            src = graph.nodes[n.inputs[0]]
            vals[n.id] = vals[src.id].reshape(src.shape).transpose(n.attrs["perm"]).reshape(-1)
        elif n.id in tmat:
            t = graph.nodes[tmat[n.id]]
            vals[n.id] = got[t.id].astype(np.float64).reshape(t.shape).transpose(t.attrs["perm"]).reshape(-1)
        else:
            vals[n.id] = got[n.id].astype(np.float64)
    expected, bound = oracle.local_reference_fused(graph, vals)
    for i in folded:
        expected[i] = bound[i] = None
    return oracle.judge_local(graph, vals, expected, bound)


def _adam_end_to_end(oracle, tr, pre, grads, state, after, after_state):
    ad = tr.ad
    feed = {**pre, **{f"g:{n}": grads[n] for n in tr.names}, **state}
    values, bounds, _ = oracle.reference_with_bounds(ad["graph"], feed)
    outs = tr.names + tr.state_names
    return oracle.judge_outputs([values[ad["outputs"][k]] for k in outs], [bounds[ad["outputs"][k]] for k in outs],
                                [{**after, **after_state}[k] for k in outs])


def test_dp_trainer_transformer_node_local(pkg, oracle, runner):
    rt, wl, dp, cg = _mods()
    s = pkg.steps
    cfg, V, B = _small_transformer(wl)
    params = s.init_params_normal(V, 0, 0.02, cfg)
    tr = dp.DPTrainer(runner, V, B, cfg, params, matmul="tiled")
    fg, gs = tr.fg, tr.gs
    grad_ids = [fg.index[gs["grads"][n]] for n in tr.names]
    lowered = cg.lower_fused(fg.graph, matmul="tiled", fold=True, keep=[tr.loss_id, *grad_ids])
    assert lowered["folded"]
    full, ids = _keep_all(rt, runner, fg.graph, lowered)
    offs, total = {}, 0
    for n in tr.names:
        offs[n] = total // 4
        total += (tr.params[n].nbytes + 255) // 256 * 256
    try:
        for t in range(3):
            x, y = wl.one_hot_batch(wl.c5_tokens(B, cfg["T"], V, seed=t), V)
            pre = tr.read(tr.names)
            state = {k: tr.adam_prog.read(tr.fa.index[tr.ad["inputs"][k]]) for k in tr.state_names}
            loss = tr.train(x, y)
            flat = tr.flat.download(tr.flat_floats)
            grads = {n: flat[offs[n]:offs[n] + pre[n].size] for n in tr.names}
            after = tr.read(tr.names)
            after_state = {k: tr.adam_prog.read(tr.fa.index[tr.ad["inputs"][k]]) for k in tr.state_names}
            # the same gradient program with every value kept, from the same parameters
            feed = {**pre, "x": x, "y": y, gs["cotangent"]: [1.0]}
            for n in fg.graph.inputs():
                full.write(n.id, feed[n.attrs["name"]])
            full.run()
            full.check_errors()
            got = {i: full.read(i) for i in ids}
            assert np.float32(loss).tobytes() == got[tr.loss_id].tobytes(), t
            for n, gid in zip(tr.names, grad_ids):
                assert np.array_equal(grads[n].view(np.uint32), got[gid].view(np.uint32)), (t, n)
            j = _node_local(pkg, oracle, fg.graph, lowered, feed, got)
            assert j["pass"], (t, {k: v for k, v in j.items() if k != "byKind"})
            assert {"matmul-epilogue", "plain"} <= set(j["byKind"])
            ja = _adam_end_to_end(oracle, tr, pre, grads, state, after, after_state)
            assert ja["pass"], (t, ja)
    finally:
        full.free()
        tr.destroy()


def test_fused_trainer_transformer_node_local(pkg, oracle, runner):
    rt, wl, _, cg = _mods()
    s = pkg.steps
    cfg, V, B = _small_transformer(wl)
    st = s.build_step3b(V, B, cfg)
    fstep = rt.fused_step(st, matmul="tiled")
    params = s.init_params_normal(V, 0, 0.02, cfg)
    state = s.adam_initial_state(st["names"], s.param_shapes(V, cfg))
    names = list(st["names"]) + list(st["stateNames"])
    tr = rt.FusedTrainer(runner, fstep, params, state)
    g = fstep["graph"]
    lowered = fstep["lowered"]
    full, ids = _keep_all(rt, runner, g, lowered)
    try:
        for t in range(3):
            x, y = wl.one_hot_batch(wl.c5_tokens(B, cfg["T"], V, seed=t), V)
            pre = tr.read(names)
            loss = tr.train(x, y)
            after = tr.read(names)
            feed = {**pre, "x": x, "y": y, st["cotangent"]: [1.0]}
            for n in g.inputs():
                full.write(n.id, feed[n.attrs["name"]])
            full.run()
            full.check_errors()
            got = {i: full.read(i) for i in ids}
            assert np.float32(loss).tobytes() == got[fstep["loss"]].tobytes(), t
            for n in names:
                assert np.array_equal(after[n].view(np.uint32), got[fstep["outputs"][n]].view(np.uint32)), (t, n)
            j = _node_local(pkg, oracle, g, lowered, feed, got)
            assert j["pass"], (t, {k: v for k, v in j.items() if k != "byKind"})
    finally:
        full.free()
        tr.destroy()
