"""The fuzz corpus (src/testing/random-graph.js v2, restated) and the fusion pass over it, pinned to
the reference's recorded m4.semantics.corpus: programs 1..2000, forward and gradient graphs, the
fused structure and bitwise float64 semantic preservation at every surviving node."""
import importlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN


def corpus_graphs(pkg, co, i):
    """The forward and gradient graphs of corpus program i with their inputs (measure-m4.js:28-40)."""
    p = co.corpus_program(i, f32=True)
    rng = pkg.rng.Rng((i * 7919 + 17) & 0xFFFFFFFF)
    inputs = {n.attrs["name"]: rng.array(pkg.ir.size(n.shape), -2, 2) for n in p.graph.inputs()}
    G = pkg.autodiff.grad(p.graph, p.outputs, [n.id for n in p.graph.inputs()])
    grad_inputs = dict(inputs)
    for k, name in enumerate(G.cotangents):
        grad_inputs[name] = rng.array(pkg.ir.size(p.graph.nodes[p.outputs[k]].shape), -1, 1)
    return [("forward", p.graph, inputs, list(p.outputs)),
            ("gradient", G.graph, grad_inputs, list(p.outputs) + list(G.grads))]


def test_corpus_structure_and_semantics_match_the_reference(pkg, oracle):
    co = importlib.import_module("tensor-compiler-webgpu_b200.corpus")
    want = json.load(open(os.path.join(GOLDEN, "pins.json")))["corpus"]
    graphs = with_fused = fused_nodes = identical = compared = 0
    by = {}
    for i in range(1, want["programs"] + 1):
        for label, g, inputs, keep in corpus_graphs(pkg, co, i):
            f = pkg.fuse.fuse(g, keep=keep)
            fz = [n for n in f.graph.nodes if n.op == "fused"]
            graphs += 1
            with_fused += bool(fz)
            fused_nodes += len(fz)
            for n in fz:
                by[n.attrs["pattern"]] = by.get(n.attrs["pattern"], 0) + 1
            s = oracle.check_semantics(g, f, inputs)
            identical += s["identical"]
            compared += s["compared"]
    assert (graphs, with_fused, fused_nodes) == (want["graphs"], want["withFused"], want["fusedNodes"])
    assert by == want["byPattern"]
    assert identical == want["identical"]
    assert compared == want["compared"]


def test_generator_is_deterministic_and_bounded(pkg):
    co = importlib.import_module("tensor-compiler-webgpu_b200.corpus")
    for i in (1, 2, 3, 10, 101, 1002):
        a, b = co.corpus_program(i, f32=True), co.corpus_program(i, f32=True)
        assert a.graph.to_json() == b.graph.to_json() and a.outputs == b.outputs
        assert all(max(abs(lo), abs(hi)) <= co.BOUND for lo, hi in (a.bounds[o] for o in a.outputs))
        assert all(pkg.ir.size(n.shape) <= co.MAX_SIZE for n in a.graph.nodes)
