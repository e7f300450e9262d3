"""Column sums fused into their elementwise producers (codegen.colsum_fusions), on the CPU: which sums
qualify, how the fused launch is shaped, and what it saves.

A sum over axis 0 whose operand is an elementwise launch's value runs inside that launch
(tcb/colsum.cuh): with the plain sum's own split, so the sum is bitwise the unfused pair's (checked on
the GPU in tests/test_gpu_colsum.py), and without storing the operand when nothing else reads it.
"""
import importlib

import pytest


@pytest.fixture(scope="module")
def cg():
    return importlib.import_module("tensor-compiler-webgpu_b200.codegen")


def test_c2_bias_gradient_runs_in_its_producer(pkg, cg):
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    W = wl.c2_graph(8192, 8192)
    f = pkg.fuse.fuse(W["graph"], keep=W["keep"])
    keep = [f.index[k] for k in W["keep"]]
    plain = cg.lower_fused(f.graph)
    fused = cg.lower_fused(f.graph, colfuse=True, keep=keep)
    cs = [l for l in fused["launches"] if l.kind == "fused-colsum"]
    assert len(cs) == 1 and len(fused["launches"]) == len(plain["launches"]) - 1
    (l,) = cs
    sum_launch = next(x for x in plain["launches"] if x.node == l.info["sum"])
    assert l.info["split"] == sum_launch.info["split"] == 37          # the plain sum's split: same partials
    assert [c.name for c in l.calls] == ["tcb_ew_colsum", "tcb_reduce_finish"]
    assert l.scratch_bytes == 37 * 8192 * 4
    # the operand (a plain neg read only by the sum) is no longer stored nor read back: 2 x 256 MiB less
    assert not l.info["write"]
    saved = sum(x.bytes for x in plain["launches"]) - sum(x.bytes for x in fused["launches"])
    assert saved == 2 * 8192 * 8192 * 4


def test_kept_or_shared_producers_are_still_stored(pkg, cg):
    g = pkg.ir.Graph()
    x = g.input("x", [300, 64])
    w = g.input("w", [64])
    y = g.tanh(g.mul(x, w))            # fused elementwise (row broadcast of w)
    s = g.sum(y, 0, True)
    z = g.exp(g.neg(y))                # another reader of y
    f = pkg.fuse.fuse(g, keep=[s, z])
    keep = [f.index[s], f.index[z]]
    low = cg.lower_fused(f.graph, colfuse=True, keep=keep)
    (l,) = [x for x in low["launches"] if x.kind == "fused-colsum"]
    assert l.info["write"] and l.nodes == [l.info["producer"], l.info["sum"]]
    assert l.node == l.info["producer"]
    fin = l.calls[1]
    assert fin.name == "tcb_reduce_finish" and fin.out_node == l.info["sum"]
    # fewer than 64 rows: one chunk, the partial sums are the result, written through p[14]
    g2 = pkg.ir.Graph()
    x2 = g2.input("x", [40, 64])
    y2 = g2.relu(x2)
    s2 = g2.sum(y2, 0, True)
    f2 = pkg.fuse.fuse(g2, keep=[y2, s2])
    (l2,) = [x for x in cg.lower_fused(f2.graph, colfuse=True, keep=[f2.index[y2], f2.index[s2]])["launches"]
             if x.kind == "fused-colsum"]
    assert l2.info["split"] == 1 and len(l2.calls) == 1 and l2.calls[0].ptr_params == ((14, l2.info["sum"]),)


def test_only_axis0_sums_of_elementwise_values_qualify(pkg, cg):
    g = pkg.ir.Graph()
    a = g.input("a", [64, 32])
    b = g.input("b", [32, 16])
    m = g.matmul(a, b)                 # a GEMM producer: not fused into
    r = g.sum(g.exp(a), 1, True)       # a row sum: the fusion pass's own rowwise kind
    c = g.sum(m, 0, True)
    one = g.sum(g.neg(g.input("v", [64, 1])), 0, True)   # a single column: not worth a column pass
    f = pkg.fuse.fuse(g, keep=[r, c, one])
    assert cg.colsum_fusions(f.graph, [f.index[k] for k in (r, c, one)]) == {}


def test_the_fused_c5_gradient_program_moves_fewer_bytes(pkg, cg):
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    s = pkg.steps
    cfg, c = wl.c5_cfg()
    gs = s.build_grad3b(c["V"], c["batch"], cfg)
    k0 = [gs["loss"], *gs["grads"].values()]
    f = pkg.fuse.fuse(gs["graph"], keep=k0)
    keep = [f.index[i] for i in k0]
    a = cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep)
    b = cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep, colfuse=True)
    cs = [l for l in b["launches"] if l.kind == "fused-colsum"]
    assert len(cs) >= 20
    assert {l.info["write"] for l in cs} == {True, False}
    assert sum(l.bytes for l in b["launches"]) < sum(l.bytes for l in a["launches"]) - 5e9


# ---------------------------------------------------------------- readers computed in their producer's pass
def test_c2_readers_run_in_their_producers(pkg, cg):
    """C2's plain launches that read a fused value (the gradient products) run inside it: 9 launches
    become 6 and the step moves 0.8 GB less."""
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    W = wl.c2_graph(8192, 8192)
    f = pkg.fuse.fuse(W["graph"], keep=W["keep"])
    keep = [f.index[k] for k in W["keep"]]
    a = cg.lower_fused(f.graph, colfuse=True, keep=keep)
    b = cg.lower_fused(f.graph, colfuse=True, mofuse=True, keep=keep)
    mo = [l for l in b["launches"] if l.kind == "fused-multi"]
    assert len(mo) == 3 and len(b["launches"]) == len(a["launches"]) - 3
    for l in mo:
        assert l.nodes == [l.info["producer"], l.info["reader"]] and l.calls[0].name == "tcb_elementwise_mo"
        assert l.calls[0].ptr_params == ((1, l.info["reader"]),)
    assert sum(l.bytes for l in a["launches"]) - sum(l.bytes for l in b["launches"]) == 3 * 8192 * 8192 * 4


def test_reader_rules(pkg, cg):
    """A reader joins its producer only when its other operands exist already, it reads the producer at
    its own index, and something kept needs it."""
    g = pkg.ir.Graph()
    x = g.input("x", [64, 32])
    p = g.exp(g.mul(x, x))                          # a fused elementwise producer
    late = g.tanh(x)                                 # kept, so stored by a launch after p's
    q_late = g.mul(p, late)                          # its other operand comes later: stays apart
    row = g.input("row", [32])
    q_ok = g.add(p, g.broadcast(row, [64, 32]))      # reads p at its own index: joins p
    dead = g.neg(p)                                  # nothing kept needs it
    f = pkg.fuse.fuse(g, keep=[p, late, q_late, q_ok])
    keep = [f.index[k] for k in (p, late, q_late, q_ok)]
    mos = cg.mo_fusions(f.graph, keep)
    pairs = {(f.origin[a], f.origin[b]) for a, b in mos.items()}
    assert (p, q_late) not in pairs and (p, dead) not in pairs
    assert any(a == p for a, _ in pairs)


def test_the_c5_gradient_program_reads_less(pkg, cg):
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    s = pkg.steps
    cfg, c = wl.c5_cfg()
    gs = s.build_grad3b(c["V"], c["batch"], cfg)
    k0 = [gs["loss"], *gs["grads"].values()]
    f = pkg.fuse.fuse(gs["graph"], keep=k0)
    keep = [f.index[i] for i in k0]
    live = set(keep)
    for n in reversed(f.graph.nodes):
        if n.id in live:
            live.update(n.inputs)

    def live_launches(low):
        return [l for l in low["launches"] if any(x in live for x in (getattr(l, "nodes", None) or [l.node]))]
    n = live_launches(cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep))
    a = live_launches(cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep, colfuse=True))
    b = live_launches(cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep, colfuse=True, mofuse=True))
    # sums in their producers' passes (22 column sums, 35 row sums), then elementwise readers too
    assert len(a) <= len(n) - 40 and sum(l.bytes for l in a) < sum(l.bytes for l in n) - 10e9
    assert len(b) <= len(a) - 20 and sum(l.bytes for l in b) < sum(l.bytes for l in a) - 8e9
    assert sum(1 for l in a if l.kind == "fused-rowsum") >= 30
