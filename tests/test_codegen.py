"""Host-side lowering: load classification, launch geometry, the byte rule, the direct cases' intended kinds."""
import importlib

import pytest


@pytest.fixture(scope="module")
def cg():
    return importlib.import_module("tensor-compiler-webgpu_b200.codegen")


def test_gather_classification(cg):
    G = cg.Gather
    assert G([8192, 8192], cg.gather_strides("broadcast", [8192, 8192], [1, 8192])).kind == "rowb"
    assert G([3, 65], cg.gather_strides("broadcast", [3, 65], [65])).P == 65
    g = G([4, 7], cg.gather_strides("broadcast", [4, 7], [4, 1]))
    assert g.kind == "colb" and g.Q == 7
    assert G([5, 5], cg.gather_strides("broadcast", [5, 5], [1])).kind == "scalar"
    assert G([2, 4, 64, 64], cg.gather_strides("broadcast", [2, 4, 64, 64], [64, 64])).P == 4096
    t = G([5, 7], cg.gather_strides("transpose", [5, 7], [7, 5], [1, 0]))
    assert t.kind == "general"
    assert G([6, 4], cg.gather_strides("reshape", [6, 4], [24])).kind == "identity"


def test_general_gather_matches_interp_index(cg):
    # the C expression evaluated in Python equals interp.js's broadcast/transpose index
    import itertools
    for out, src, op, perm in (([2, 4, 3, 5], [2, 1, 3, 1], "broadcast", None), ([2, 3, 4], [3, 4, 2], "transpose", [2, 0, 1])):
        g = cg.Gather(out, cg.gather_strides(op, out, src, perm))
        expr = g.expr("i", "u64").replace("(u64)", "").replace("ull", "").replace("/", "//")
        n = 1
        for d in out:
            n *= d
        from math import prod
        for i in range(n):
            coords = []
            rem = i
            for d in reversed(out):
                coords.append(rem % d)
                rem //= d
            coords.reverse()
            st = [prod(src[k + 1:]) for k in range(len(src))]
            if op == "broadcast":
                lead = len(out) - len(src)
                want = sum(coords[lead + k] * st[k] for k in range(len(src)) if src[k] != 1)
            else:
                want = sum(coords[d] * st[perm[d]] for d in range(len(out)))
            assert eval(expr, {"i": i}) == want


def test_rowwise_geometry(cg):
    geo = cg.rowwise_geometry(65536, 4096, 1)
    assert geo["vec"] == 4 and geo["tpr"] == 256 and geo["items"] == 16 and geo["cache"]
    geo = cg.rowwise_geometry(64, 10, 1)
    assert geo["vec"] == 1 and geo["tpr"] == 32 and geo["groups"] == 8
    geo = cg.rowwise_geometry(1, 4097, 2)
    assert geo["vec"] == 1 and geo["tpr"] == 512 and geo["slots"] == 9


def test_byte_rule_counts_distinct_operands_once(pkg, cg):
    g = pkg.ir.Graph()
    x = g.input("x", [100])
    y = g.mul(x, x)
    low = cg.lower(g)
    assert low["launches"][0].bytes == 100 * 4 + 100 * 4


def test_direct_cases_fuse_to_their_intended_kind(pkg):
    cases = importlib.import_module("tensor-compiler-webgpu_b200.cases").fused_direct_cases()
    assert len(cases) == 100
    for c in cases:
        f = pkg.fuse.fuse(c["graph"])
        fused = [n for n in f.graph.nodes if n.op == "fused"]
        assert sorted({n.attrs["kind"] for n in fused}) == [c["kind"]], c["name"]
        assert sorted({n.attrs["pattern"] for n in fused}) == [c["pattern"]], c["name"]


def test_fused_launches_replace_the_plain_ones(pkg, cg):
    w = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    W = w.c2_graph(64, 64)
    f = pkg.fuse.fuse(W["graph"], keep=W["keep"])
    fused = cg.lower_fused(f.graph)["launches"]
    plain = cg.lower(W["graph"])["launches"]
    assert len(fused) < len(plain)
    assert sum(1 for l in fused if l.kind == "fused-elementwise") == 4


def test_transpose_folding_picks_only_gemm_operand_transposes(pkg, cg):
    g = pkg.ir.Graph()
    a = g.input("a", [64, 96])
    w = g.input("w", [48, 96])
    wt = g.transpose(w, [1, 0])           # [96, 48], read only as a GEMM operand: folded
    g.matmul(a, wt)
    u = g.transpose(a, [1, 0])            # [96, 64], also read by an elementwise op: kept
    g.add(g.matmul(u, a), g.const(1.0))
    g.exp(u)
    folds = cg.foldable_transposes(g, "tiled")
    assert folds == {wt}
    low = cg.lower(g, matmul="tiled", fold=True)
    assert wt not in {l.node for l in low["launches"]}
    mm = [l for l in low["launches"] if l.op == "matmul"]
    assert [l.info.get("b_t") for l in mm] == [True, False]
    assert mm[0].inputs == [a, w]
    assert cg.foldable_transposes(g, "naive") == set()   # CUDA-core path: nothing folds
