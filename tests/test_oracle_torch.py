"""A second, independent float64 oracle: PyTorch, op by op, against the C oracle and the host autodiff.

The reference keeps PyTorch as its independent checker (oracle/torch_golden.py:26-70: every graph
rebuilt op for op in float64, gradients by autograd).  Its golden file pins the C oracle on 112
cases (tests/test_oracle_golden.py); this test restates that checker and runs it live on the
restated fuzz corpus (random-graph.js v2), a different population of graphs:

* forward values: every node of each program's forward graph, C oracle vs PyTorch float64;
* gradients: the C oracle evaluating the host autodiff's gradient graph vs PyTorch autograd on the
  forward graph, for the same cotangents.

Metric v2 at 1e-12 (src/testing/golden.js:36-49), as the golden pins use.
"""
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")

F64 = torch.float64
SAMPLE = list(range(1, 2001, 20)) + list(range(2, 2001, 20))   # 200 corpus programs, general and targeted


def torch_run(graph, leaves):
    """The graph in PyTorch float64, node by node (the checker of oracle/torch_golden.py:26-70)."""
    vals = []
    for n in graph.nodes:
        ins = [vals[i] for i in n.inputs]
        a = n.attrs
        op = n.op
        if op == "input":
            v = leaves[a["name"]]
        elif op == "const":
            c = a["value"]
            v = (torch.full(list(n.shape), float(c), dtype=F64) if isinstance(c, (int, float))
                 else torch.tensor(c, dtype=F64).reshape(list(n.shape)))
        elif op in ("add", "sub", "mul", "div"):
            v = {"add": torch.add, "sub": torch.sub, "mul": torch.mul, "div": torch.div}[op](ins[0], ins[1])
        elif op == "neg":
            v = torch.neg(ins[0])
        elif op == "exp":
            v = torch.exp(ins[0])
        elif op == "log":
            v = torch.log(ins[0])
        elif op == "relu":
            v = torch.relu(ins[0])
        elif op == "tanh":
            v = torch.tanh(ins[0])
        elif op == "sqrt":
            v = torch.sqrt(ins[0])
        elif op == "step":
            v = (ins[0] > 0).to(F64)
        elif op == "stopGradient":
            v = ins[0].detach()
        elif op == "matmul":
            v = torch.matmul(ins[0], ins[1])
        elif op == "sum":
            v = torch.sum(ins[0], dim=a["axis"], keepdim=a["keepDims"])
        elif op == "max":
            v = torch.amax(ins[0], dim=a["axis"], keepdim=a["keepDims"])
        elif op == "broadcast":
            v = torch.broadcast_to(ins[0], list(a["shape"]))
        elif op == "reshape":
            v = torch.reshape(ins[0], list(a["shape"]))
        elif op == "transpose":
            v = torch.permute(ins[0], list(a["perm"]))
        else:
            raise ValueError(f"unknown op {op}")
        assert list(v.shape) == list(n.shape), (op, list(v.shape), list(n.shape))
        vals.append(v)
    return vals


def _program(pkg, co, i):
    """Corpus program i with the inputs and cotangents test_corpus.py draws for it."""
    p = co.corpus_program(i, f32=True)
    rng = pkg.rng.Rng((i * 7919 + 17) & 0xFFFFFFFF)
    inputs = {n.attrs["name"]: rng.array(pkg.ir.size(n.shape), -2, 2) for n in p.graph.inputs()}
    cots = [rng.array(pkg.ir.size(p.graph.nodes[o].shape), -1, 1) for o in p.outputs]
    return p, inputs, cots


def test_c_oracle_matches_torch_float64_on_the_corpus(pkg, oracle):
    co = importlib.import_module("tensor-compiler-webgpu_b200.corpus")
    worst, checked = 0.0, 0
    for i in SAMPLE:
        p, inputs, _ = _program(pkg, co, i)
        ours = oracle.evaluate(p.graph, inputs)
        leaves = {n.attrs["name"]: torch.tensor(np.asarray(inputs[n.attrs["name"]], np.float64),
                                                dtype=F64).reshape(list(n.shape)) for n in p.graph.inputs()}
        ref = torch_run(p.graph, leaves)
        for n in p.graph.nodes:
            s = oracle.tensor_score(ours[n.id], ref[n.id].detach().numpy())
            worst = max(worst, s)
            assert s <= 1, (i, n.id, n.op, s)
            checked += 1
    assert checked > 1000


def test_host_autodiff_matches_torch_autograd_on_the_corpus(pkg, oracle):
    co = importlib.import_module("tensor-compiler-webgpu_b200.corpus")
    compared = 0
    for i in SAMPLE:
        p, inputs, cots = _program(pkg, co, i)
        ins = p.graph.inputs()
        G = pkg.autodiff.grad(p.graph, p.outputs, [n.id for n in ins])
        feed = dict(inputs)
        for k, name in enumerate(G.cotangents):
            feed[name] = cots[k]
        ours = oracle.evaluate(G.graph, feed)
        leaves = {n.attrs["name"]: torch.tensor(np.asarray(inputs[n.attrs["name"]], np.float64), dtype=F64)
                  .reshape(list(n.shape)).requires_grad_(True) for n in ins}
        vals = torch_run(p.graph, leaves)
        outs = [vals[o] for o in p.outputs]
        seeds = [torch.tensor(np.asarray(c, np.float64), dtype=F64).reshape(o.shape) for c, o in zip(cots, outs)]
        wrt = [leaves[n.attrs["name"]] for n in ins]
        live = [(o, sd) for o, sd in zip(outs, seeds) if o.requires_grad]  # a step / stopGradient output has none
        if live:
            grads = torch.autograd.grad([o for o, _ in live], wrt, grad_outputs=[sd for _, sd in live],
                                        allow_unused=True)
        else:
            grads = [None] * len(wrt)
        for k, n in enumerate(ins):
            g = grads[k]
            ref = np.zeros(pkg.ir.size(n.shape)) if g is None else g.detach().numpy().reshape(-1)
            s = oracle.tensor_score(ours[G.grads[k]], ref)
            assert s <= 1, (i, n.attrs["name"], s)
            compared += 1
    assert compared > 100
