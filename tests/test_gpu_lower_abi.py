"""The whole path through the C ABI alone, on the B200: graph JSON -> tc_lower_json -> tc_lowered_run or
tc_program_*, with no Python host between the caller and the library.

* A plain C program (tests/c/run_graph.c, built here with gcc against include/tcb200.h) lowers the C2
  chain (forward + backward, fused) and a C3 matmul epilogue on the tcgen05 path from their JSON, runs
  them with canary-padded buffers and writes every node's value: bit for bit the Python host's
  GpuRunner.run of its own lowering, and within 2E of the float64 oracle.
* Through ctypes only (the library loaded by path, every signature declared here): the resident program
  of the C1 training step (Adam, parameters and state fed back on the device, one captured CUDA graph)
  over three steps against the Python host's FusedTrainer, and the transformer's gradient program as the
  data-parallel trainer lowers it (folded transposes, fused column sums), bit for bit.
"""
import ctypes
import importlib
import json
import os
import subprocess
import tempfile

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

PKG_DIR = os.path.join(ROOT, "tensor-compiler-webgpu_b200")


def _lib():
    lib = ctypes.CDLL(os.path.join(PKG_DIR, "libtcb200.so"))
    P, I, U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64
    sigs = {"tc_last_error": ([], ctypes.c_char_p), "tc_open": ([I, ctypes.POINTER(P)], I), "tc_close": ([P], I),
            "tc_lower_json": ([ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(P)], I),
            "tc_lowered_free": ([P], I),
            "tc_program_create": ([P, P, ctypes.POINTER(ctypes.c_int32), I, ctypes.POINTER(ctypes.c_int32), I, I,
                                   ctypes.POINTER(P)], I),
            "tc_program_write": ([P, I, P, U64], I), "tc_program_read": ([P, I, P, U64], I),
            "tc_program_run": ([P], I), "tc_program_check": ([P], I), "tc_program_free": ([P], I),
            "tc_program_launch_count": ([P, ctypes.POINTER(I)], I)}
    for name, (args, res) in sigs.items():
        f = getattr(lib, name)
        f.argtypes, f.restype = args, res
    return lib


def _ok(lib, st):
    assert st == 0, lib.tc_last_error().decode()


@pytest.fixture(scope="module")
def run_graph():
    exe = os.path.join(tempfile.mkdtemp(prefix="tcb_c_"), "run_graph")
    subprocess.run(["gcc", "-O2", "-o", exe, os.path.join(ROOT, "tests", "c", "run_graph.c"),
                    "-I" + os.path.join(ROOT, "include"), "-L" + PKG_DIR, "-ltcb200", "-Wl,-rpath," + PKG_DIR],
                   check=True)
    return exe


def _c_run(exe, fgraph, opts, inputs):
    d = tempfile.mkdtemp(prefix="tcb_run_")
    paths = [os.path.join(d, n) for n in ("g.json", "o.json", "in.bin", "out.bin")]
    with open(paths[0], "w") as f:
        json.dump(fgraph.to_json(), f)
    with open(paths[1], "w") as f:
        json.dump(opts, f)
    with open(paths[2], "wb") as f:
        for n in fgraph.nodes:
            if n.op == "input":
                f.write(np.asarray(inputs[n.attrs["name"]], np.float32).reshape(-1).tobytes())
    p = subprocess.run([exe, *paths], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr
    out = np.fromfile(paths[3], dtype=np.float32)
    vals, off = [], 0
    for n in fgraph.nodes:
        k = int(np.prod(n.shape, dtype=np.int64))
        vals.append(out[off:off + k])
        off += k
    assert off == out.size
    return vals, json.loads(p.stdout)


@pytest.mark.parametrize("case", ["c2", "c3"])
def test_c_host_lowers_and_runs_a_graph_from_json(pkg, oracle, runner, run_graph, case):
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    if case == "c2":
        W = wl.c2_graph(257, 1000)
        inputs, matmul = wl.c2_inputs(W), "naive"
    else:
        W = wl.c3_graph(300, 256, 384, "tanh")
        inputs, matmul = wl.c3_inputs(300, 256, 384), "tiled"
    values, bounds, rounded = oracle.reference_with_bounds(W["graph"], inputs)
    fused = pkg.fuse.fuse(W["graph"], keep=W["keep"])
    got, info = _c_run(run_graph, fused.graph, {"fused": True, "matmul": matmul}, rounded)
    py = runner.run(fused.graph, cg.lower_fused(fused.graph, matmul=matmul), rounded)
    assert info["launches"] == len(cg.lower_fused(fused.graph, matmul=matmul)["launches"])
    for n in fused.graph.nodes:
        assert np.array_equal(got[n.id].view(np.uint32), py["values"][n.id].view(np.uint32)), n.id
    j = oracle.judge_fused(fused, got, values, bounds)
    assert j["pass"], j["first"]


def _program(lib, ctx, fgraph, opts, keep, feedback=()):
    low = ctypes.c_void_p()
    _ok(lib, lib.tc_lower_json(json.dumps(fgraph.to_json()).encode(), json.dumps(opts).encode(), ctypes.byref(low)))
    k = (ctypes.c_int32 * max(1, len(keep)))(*keep)
    fb = [v for pair in feedback for v in pair]
    f = (ctypes.c_int32 * max(1, len(fb)))(*fb)
    prog = ctypes.c_void_p()
    _ok(lib, lib.tc_program_create(ctx, low, k, len(keep), f, len(feedback), 1, ctypes.byref(prog)))
    return low, prog


def _write(lib, prog, nid, arr):
    a = np.ascontiguousarray(np.asarray(arr, np.float32).reshape(-1))
    _ok(lib, lib.tc_program_write(prog, nid, a.ctypes.data, a.size))


def _read(lib, prog, nid, n):
    a = np.empty(n, np.float32)
    _ok(lib, lib.tc_program_read(prog, nid, a.ctypes.data, n))
    return a


def test_resident_training_step_through_the_c_abi(pkg, runner):
    """The C1 MLP step with Adam as a resident program created, fed and replayed through the C ABI only:
    three steps, loss and every parameter and state tensor bitwise those of the Python FusedTrainer."""
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    s = pkg.steps
    step = s.build_mlp_step(wl.C1_DIMS, 64, opt=s.ADAM, hidden="tanh")
    fstep = rt.fused_step(step, matmul="tiled")
    data = wl.c1_inputs(64)
    params = {k: data[k] for k in s.PARAMS}
    state = s.mlp_initial_state(s.ADAM, wl.C1_DIMS)
    names = list(params) + list(state)
    g = fstep["graph"]
    keep = [fstep["loss"], *[fstep["outputs"][n] for n in names]]
    feedback = [(fstep["outputs"][n], fstep["inputs"][n]) for n in names]
    lib = _lib()
    ctx = ctypes.c_void_p()
    _ok(lib, lib.tc_open(0, ctypes.byref(ctx)))
    low, prog = _program(lib, ctx, g, {"fused": True, "matmul": "tiled"}, keep, feedback)
    tr = rt.FusedTrainer(runner, fstep, params, state)
    try:
        cot = g.input_id(step["cotangent"])
        _write(lib, prog, cot, [1.0])
        for n, v in {**params, **state}.items():
            _write(lib, prog, fstep["inputs"][n], v)
        size = lambda nid: int(np.prod(g.nodes[nid].shape, dtype=np.int64))
        for it in range(3):
            x = data["x"] if it % 2 == 0 else data["x"][::-1].copy()
            _write(lib, prog, fstep["inputs"]["x"], x)
            _write(lib, prog, fstep["inputs"]["y"], data["y"])
            _ok(lib, lib.tc_program_run(prog))
            _ok(lib, lib.tc_program_check(prog))
            loss = _read(lib, prog, fstep["loss"], 1)
            want = tr.train(x, data["y"])
            assert np.float32(want).tobytes() == loss.tobytes(), it
        ref = tr.read(names)
        for n in names:
            got = _read(lib, prog, fstep["inputs"][n], size(fstep["inputs"][n]))
            assert np.array_equal(got.view(np.uint32), ref[n].view(np.uint32)), n
    finally:
        tr.destroy()
        lib.tc_program_free(prog)
        lib.tc_lowered_free(low)
        lib.tc_close(ctx)


def test_transformer_gradient_program_through_the_c_abi(pkg, runner):
    """The gradient program of the data-parallel trainer (tiled GEMMs, folded transposes, fused column
    sums) lowered and made resident through the C ABI: loss and every gradient bitwise the trainer's."""
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    dp = importlib.import_module("tensor-compiler-webgpu_b200.dp")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=64, L=2, H=4, ff=128, T=32, batch=4)
    V, B = c["V"], c["batch"]
    params = s.init_params_normal(V, 0, 0.02, cfg)
    tr = dp.DPTrainer(runner, V, B, cfg, params)
    fg, gs = tr.fg, tr.gs
    grad_ids = [fg.index[gs["grads"][n]] for n in tr.names]
    keep = [tr.loss_id, *grad_ids]
    lib = _lib()
    ctx = ctypes.c_void_p()
    _ok(lib, lib.tc_open(0, ctypes.byref(ctx)))
    low, prog = _program(lib, ctx, fg.graph, {"fused": True, "matmul": "tiled", "fold": True, "colfuse": True,
                                              "keep": keep}, keep)
    try:
        x, y = wl.one_hot_batch(wl.c5_tokens(B, cfg["T"], V, seed=3), V)
        feed = {**params, "x": x, "y": y, gs["cotangent"]: [1.0]}
        for n in fg.graph.inputs():
            _write(lib, prog, n.id, feed[n.attrs["name"]])
        _ok(lib, lib.tc_program_run(prog))
        _ok(lib, lib.tc_program_check(prog))
        tr.train(x, y)
        flat = tr.flat.download(tr.flat_floats)
        off = 0
        for n, gid in zip(tr.names, grad_ids):
            k = int(np.prod(fg.graph.nodes[gid].shape, dtype=np.int64))
            got = _read(lib, prog, gid, k)
            assert np.array_equal(got.view(np.uint32), flat[off:off + k].view(np.uint32)), n
            off += (k * 4 + 255) // 256 * 64
        assert _read(lib, prog, tr.loss_id, 1).tobytes() == tr.grad_prog.read(tr.loss_id).tobytes()
    finally:
        tr.destroy()
        lib.tc_program_free(prog)
        lib.tc_lowered_free(low)
        lib.tc_close(ctx)
