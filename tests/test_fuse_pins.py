"""The host fusion pass against the reference's recorded structure (golden/measurements.json m4).

Golden config 1 (V=16, batch 4): forward 212 -> 48 launches, step 1308 -> 450,
each pattern count, and bitwise float64 semantic preservation at every
surviving node (src/fusion/fuse.js:311-330; 84 and 556 nodes compared).
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN


def _pins():
    with open(os.path.join(GOLDEN, "pins.json")) as f:
        return json.load(f)


def _model_graphs(pkg):
    s = pkg.steps
    pins = _pins()["goldenConfig"]
    V, B = pins["V"], pins["batch"]
    T = s.CONFIG["T"]
    rng = pkg.rng.Rng(7)
    seqs = [[rng.int(0, V - 1) for _ in range(T + 1)] for _ in range(B)]
    x, y = s.encode_batch(seqs, V, T)
    params = s.init_params(V, pins["seed"])
    f = s.build_forward(V, B)
    st = s.build_step3b(V, B)
    state = s.adam_initial_state(st["names"], s.param_shapes(V))
    return [
        ("forward", f["graph"], {**params, "x": x, "y": y}, [f["logits"], f["loss"]]),
        ("step", st["graph"], {**params, **state, "x": x, "y": y, st["cotangent"]: [1.0]},
         [st["loss"], st["logits"], *st["outputs"].values()]),
    ]


def test_model_fusion_structure_matches_reference(pkg):
    pins = {p["graph"]: p for p in _pins()["fusion"]}
    for label, graph, _, keep in _model_graphs(pkg):
        f = pkg.fuse.fuse(graph, keep=keep)
        summary = pkg.fuse.fusion_summary(graph, f)
        want = pins[label]
        assert summary["launchesBefore"] == want["launchesBefore"], label
        assert summary["launchesAfter"] == want["launchesAfter"], label
        assert summary["byPattern"] == want["byPattern"], label
        epi = [g for g in f.groups if g.kind == "epilogue"]
        act = sum(1 for g in epi if any(graph.nodes[i].op in ("tanh", "relu") for i in g.members))
        assert len(epi) == want["epilogues"] and act == want["epiloguesWithActivation"], label


def test_model_fusion_preserves_semantics_bitwise(pkg, oracle):
    pins = {p["graph"]: p for p in _pins()["semanticsModel"]}
    for label, graph, inputs, keep in _model_graphs(pkg):
        f = pkg.fuse.fuse(graph, keep=keep)
        s = oracle.check_semantics(graph, f, inputs)
        assert s["identical"], (label, s["first"])
        assert s["compared"] == pins[label]["compared"], label


def test_pass_sabotage_breaks_the_model(pkg):
    # golden/measurements.json m4.passSabotage.model: the sabotaged pass throws on both graphs
    for label, graph, _, keep in _model_graphs(pkg):
        with pytest.raises(RuntimeError, match="used before it is built"):
            pkg.fuse.fuse(graph, keep=keep, sabotage="fusion-absorbs-shared")
