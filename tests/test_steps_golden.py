"""The step builders (steps.py) on the float64 oracle against the reference's PyTorch training goldens.

* MLP (src/train/step.js, the milestone-3 step): golden/train-spec-m3.json's 8 runs (SGD and Adam, 50
  steps each, 8 -> 16 -> 4 relu, batch 32) trained on the oracle from the recorded initial parameters
  and batch schedule; the loss and every parameter after every step against golden/torch-train-m3.json
  at metric v2 1e-8 (src/train/verify-cpu.js:9-28).
* Transformer (src/m3b/model.js, step.js, adam.js): golden/spec-m3b.json's 4 synthetic golden runs.  At
  initialisation the loss and logits of every run, and golden-seed1's gradients of every parameter,
  against golden/torch-m3b.{json,f64} at TAU1 = 1e-10; then 20 Adam steps, the loss and k = 4 seeded
  projections of every parameter after every step at TAU2 = 1e-8, and golden-seed1's parameters after
  step 20 elementwise at TAU2 (src/m3b/verify-cpu.js:11-12, :64-113).  The initial parameters and the
  projection vectors are pinned first by the spec's own SHA-256 hashes of their float64 bytes
  (src/m3b/spec.js:14-26).  The text case needs the book it was drawn from and is left out.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

TRAIN_TOL = 1e-8   # src/train/verify-cpu.js:9
TAU1, TAU2 = 1e-10, 1e-8   # src/m3b/verify-cpu.js:11-12


def _load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def v2(ours, ref, tau):
    """Metric v2 at tolerance tau (src/m3b/verify-cpu.js:15-24)."""
    ours = np.asarray(ours, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    atol = tau * max(1.0, float(np.abs(ref).max()) if ref.size else 0.0)
    d = np.abs(ours - ref)
    r = d / (atol + tau * np.abs(ref))
    return float(np.where(np.isnan(d), np.inf, r).max()) if r.size else 0.0


# ---------------------------------------------------------------- MLP (milestone 3)
def _gather(data, idx, features, classes):
    """src/train/data.js:76-83."""
    x = np.asarray(data["x"], np.float64).reshape(-1, features)[idx].reshape(-1)
    y = np.zeros((len(idx), classes))
    y[np.arange(len(idx)), np.asarray(data["y"])[idx]] = 1
    return x, y.reshape(-1)


def test_mlp_step_trains_like_torch(pkg, oracle):
    spec = _load("train_m3.json")
    params_ref = np.load(os.path.join(GOLDEN, "train_m3_params.npz"))
    s = pkg.steps
    dims = spec["dims"]
    assert spec["dtype"] == "float64" and len(spec["configs"]) == 8
    for k, cfg in enumerate(spec["configs"]):
        step = s.build_mlp_step(dims, cfg["batch"], opt=cfg["optimizer"])
        params = {p: np.asarray(cfg["init"][p], np.float64) for p in s.PARAMS}
        state = {n: np.asarray(v, np.float64) for n, v in s.mlp_initial_state(cfg["optimizer"], dims).items()}
        worst = 0.0
        for t in range(cfg["steps"]):
            x, y = _gather(spec["synthetic"]["train"], cfg["schedule"][t], dims["inputs"], dims["classes"])
            vals = oracle.evaluate(step["graph"], {**params, **state, "x": x, "y": y, step["cotangent"]: [1.0]})
            worst = max(worst, v2([vals[step["loss"]][0]], [spec["losses"][k][t]], TRAIN_TOL))
            params = {p: vals[step["outputs"][p]] for p in s.PARAMS}
            state = {n: vals[step["outputs"][n]] for n in state}
            for p in s.PARAMS:
                worst = max(worst, v2(params[p], params_ref[p][k, t], TRAIN_TOL))
        assert worst <= 1, (cfg["name"], worst)


# ---------------------------------------------------------------- transformer (milestone 3b)
def _fnv(name):
    h = 0x811C9DC5
    for ch in name:
        h = ((h ^ ord(ch)) * 0x01000193) & 0xFFFFFFFF
    return h


def projection_vector(pkg, name, n, k):
    """The k-th projection vector of a parameter: uniform in [-1, 1] (src/m3b/config.js:14-24)."""
    return np.asarray(pkg.rng.Rng((_fnv(name) + 7919 * k) & 0xFFFFFFFF).array(n, -1, 1), np.float64)


def _sha_f64(arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.asarray(a, "<f8").tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def m3b(pkg):
    spec = _load("m3b.json")
    blob = np.load(os.path.join(GOLDEN, "m3b_blob.npz"))
    s = pkg.steps
    cfg = s.make_config(**{k: spec["config"][k] for k in ("T", "d", "H", "L", "ff")})
    assert cfg["eps"] == spec["config"]["eps"] and cfg["mask"] == spec["config"]["mask"]
    return spec, blob, cfg


def test_transformer_init_and_projection_hashes(pkg, m3b):
    spec, _, cfg = m3b
    s = pkg.steps
    V = spec["synthetic"]["vocab"]
    assert [p["name"] for p in spec["paramOrder"]] == s.param_names(V, cfg)
    for g in spec["golden"]:
        p = s.init_params(g["V"], g["seed"], cfg)
        assert _sha_f64([p[n] for n in s.param_names(g["V"], cfg)]) == g["initSha"], g["name"]
    shapes = s.param_shapes(V, cfg)
    vecs = [projection_vector(pkg, n, int(np.prod(shapes[n])), k) for n in s.param_names(V, cfg)
            for k in range(spec["projections"]["k"])]
    assert _sha_f64(vecs) == spec["projections"]["sha256"]


def test_transformer_at_init_matches_torch(pkg, oracle, m3b):
    spec, blob, cfg = m3b
    s = pkg.steps
    syn = spec["synthetic"]["train"]
    for k, g in enumerate(spec["golden"]):
        V, B = g["V"], g["batch"]
        params = s.init_params(V, g["seed"], cfg)
        x, y = s.encode_batch([syn[i] for i in g["schedule"][0]], V, cfg["T"])
        gs = s.build_grad3b(V, B, cfg)
        vals = oracle.evaluate(gs["graph"], {**params, "x": x, "y": y, gs["cotangent"]: [1.0]})
        assert spec["init"][k]["name"] == g["name"]
        assert v2([vals[gs["loss"]][0]], [spec["init"][k]["loss"]], TAU1) <= 1, g["name"]
        assert v2(vals[gs["logits"]], blob[f"init/{g['name']}/logits"], TAU1) <= 1, g["name"]
        if k == 0:
            for n in gs["names"]:
                assert v2(vals[gs["grads"][n]], blob[f"init/{g['name']}/grad/{n}"], TAU1) <= 1, (g["name"], n)


def _projection_score(ours, r, ref_proj, tau):
    """src/m3b/verify-cpu.js:35-42."""
    atol = tau * max(1.0, float(np.abs(ours).max()))
    p = float(np.dot(r, ours))
    allow = float(np.sum(np.abs(r) * (atol + tau * np.abs(ours))))
    return abs(p - ref_proj) / allow


def test_transformer_training_matches_torch(pkg, oracle, m3b):
    spec, blob, cfg = m3b
    s = pkg.steps
    syn = spec["synthetic"]["train"]
    opt = spec["optimizer"]
    kproj = spec["projections"]["k"]
    V0 = spec["synthetic"]["vocab"]
    shapes = s.param_shapes(V0, cfg)
    r = {n: [projection_vector(pkg, n, int(np.prod(shapes[n])), j) for j in range(kproj)]
         for n in s.param_names(V0, cfg)}
    for k, g in enumerate(spec["golden"]):
        V, B = g["V"], g["batch"]
        ref = spec["training"][k]
        assert ref["name"] == g["name"]
        st = s.build_step3b(V, B, cfg, opt)
        params = {n: np.asarray(v, np.float64) for n, v in s.init_params(V, g["seed"], cfg).items()}
        state = {n: np.asarray(v, np.float64) for n, v in s.adam_initial_state(st["names"], s.param_shapes(V, cfg)).items()}
        worst_loss = worst_proj = 0.0
        for t in range(g["steps"]):
            x, y = s.encode_batch([syn[i] for i in g["schedule"][t]], V, cfg["T"])
            vals = oracle.evaluate(st["graph"], {**params, **state, "x": x, "y": y, st["cotangent"]: [1.0]})
            worst_loss = max(worst_loss, v2([vals[st["loss"]][0]], [ref["losses"][t]], TAU2))
            params = {n: vals[st["outputs"][n]] for n in st["names"]}
            state = {n: vals[st["outputs"][n]] for n in state}
            for n in st["names"]:
                for j in range(kproj):
                    worst_proj = max(worst_proj, _projection_score(params[n], r[n][j], ref["projections"][t][n][j], TAU2))
        assert worst_loss <= 1 and worst_proj <= 1, (g["name"], worst_loss, worst_proj)
        if k == 0:
            for n in st["names"]:
                assert v2(params[n], blob[f"train/{g['name']}/final/{n}"], TAU2) <= 1, (g["name"], n)
