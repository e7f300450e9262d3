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


@pytest.mark.parametrize("shape", [(1, 4096, 4096, 4096), (1, 16384, 1024, 4096), (198, 128, 256, 128),
                                   (1, 5120, 256, 1024), (1, 2432, 128, 2048), (2048, 256, 64, 256),
                                   (1, 256, 131072, 768), (3, 300, 96, 500), (1, 16384, 256, 256),
                                   (1, 2560, 1024, 512), (1, 256, 16384, 1024), (1, 3456, 512, 2048),
                                   (1, 5760, 512, 1024), (1, 16384, 256, 1024), (256, 256, 256, 64)])
def test_gemm_last_wave_plan(cg, shape):
    """The persistent GEMM's unit schedule: every (tile, k-block) is covered exactly once, the last wave
    is split only when it would leave at least half the CTAs idle, and no CTA gets more than one
    unit beyond the full waves."""
    batch, M, K, N = shape
    bn = cg.gemm_bn(N)
    bk = cg.gemm_bk(bn)
    splitk, _ = cg.splitk_plan(batch, M, K, N, bn)
    grid, tail, rem_plan, tail_off, end = cg.tail_plan(batch, M, K, N, bn, bk, splitk)
    tiles = batch * -(-M // cg.GEMM_BM) * -(-N // bn) * splitk
    if tiles < cg.SM_COUNT and splitk == 1:
        assert grid == tiles * tail                  # every tile split, one K range per CTA
    else:
        assert grid == min(cg.SM_COUNT, tiles)
    assert splitk == 1 or tiles // splitk <= cg.SM_COUNT // 9
    kb_all = cg._kpad(K) // bk
    rem = tiles % grid if tail > 1 else 0
    u_full = tiles - rem
    units = u_full + rem * tail
    covered = {}
    for u in range(units):
        if u < u_full:
            t, kb0, kb1 = u, 0, kb_all
        else:
            v = u - u_full
            t, p = u_full + v // tail, v % tail
            kb0, kb1 = p * kb_all // tail, (p + 1) * kb_all // tail
        assert kb1 > kb0
        covered.setdefault(t, []).append((kb0, kb1))
    assert sorted(covered) == list(range(tiles))
    for rngs in covered.values():
        assert rngs[0][0] == 0 and rngs[-1][1] == kb_all
        assert all(a[1] == b[0] for a, b in zip(rngs, rngs[1:]))
    per_cta = [len(range(c, units, grid)) for c in range(grid)]
    assert max(per_cta) - min(per_cta) <= 1
    if tail > 1:
        assert splitk == 1 and 2 * rem <= grid and kb_all // tail >= 4
        assert rem_plan == rem and tail_off >= cg.ctrl_bytes(rem)
        assert end == tail_off + rem * tail * cg.GEMM_BM * bn * 4
        if tiles >= cg.SM_COUNT:
            assert kb_all >= cg.TAIL_MIN_KB        # a last wave is split only with a long enough K
    elif tiles >= cg.SM_COUNT and splitk == 1:
        r = tiles % grid
        assert not (r and 2 * r <= grid and kb_all >= cg.TAIL_MIN_KB and min(grid // r, kb_all // 4, 8) >= 2)


def test_batch_small_launches_keeps_dependencies():
    """Small launches are hoisted to just after their last producer and same-source ones that land on
    one slot are batched; every value is still produced before it is read, and large launches keep their
    relative order."""
    import importlib
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    cgm = importlib.import_module("tensor-compiler-webgpu_b200.codegen")

    class L:
        def __init__(self, node, inputs, code, n=1000):
            self.node, self.inputs, self.code = node, inputs, code
            self.calls = [cgm.KernelCall("tcb_elementwise", (4, 1, 1), (256, 1, 1), 0, [n])]
            self.scratch_bytes, self.pattern, self.kind, self.bytes, self.info = 0, None, "e", 0, {}

    # an Adam-like interleaving: per parameter j, m_j = M(g_j), v_j = V(g_j), p_j = P(m_j, v_j); then a
    # large launch X reading p_0 and a small Q reading X
    seq = []
    for j in range(3):
        seq += [L(100 + j, [j], "M"), L(200 + j, [j], "V"), L(300 + j, [100 + j, 200 + j], "P")]
    seq += [L(400, [300], "X", n=1 << 22), L(401, [400], "M"), L(402, [5], "M")]
    out = rt.batch_small_launches(seq, lambda i: i)
    got = [sorted(getattr(x, "nodes", [x.node])) for x in out]
    assert got == [[100, 101, 102, 402], [200, 201, 202], [300, 301, 302], [400], [401]]
    pos = {n: k for k, x in enumerate(out) for n in getattr(x, "nodes", [x.node])}
    for x in out:
        for i in x.inputs:
            if i in pos:
                assert pos[i] < pos[x.node], (i, x.node)


def test_c5_step_roofline(pkg, cg):
    """bench.step_roofline on the C5 programs: the GEMMs' useful flops are the model's (about 2.9
    TFLOP per 131,072-token step) and the ideal step lies between the pure-HBM and pure-tensor bounds."""
    import importlib
    import sys
    import os
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    bench = importlib.import_module("bench")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    cfg, c = wl.c5_cfg(batch=512)
    V = c["V"]
    gs = pkg.steps.build_grad3b(V, 512, cfg)
    names = gs["names"]
    keep = [gs["loss"], *[gs["grads"][n] for n in names]]
    fg = pkg.fuse.fuse(gs["graph"], keep=keep)
    grad_ids = [fg.index[gs["grads"][n]] for n in names]
    low = cg.lower_fused(fg.graph, matmul="tiled", fold=True, keep=[fg.index[gs["loss"]], *grad_ids])
    sr = bench.step_roofline(low["launches"], 6558.1, 1396.5 / 6)
    assert 2.8 < sr["matmul_tflop"] < 3.0
    assert sr["hbm_ms"] > 0 and sr["gemm_ms"] >= sr["matmul_tflop"] / (1396.5 / 6) * 1e3 - 1e-6
    assert abs(sr["ideal_ms"] - sr["gemm_ms"] - sr["hbm_ms"]) < 1e-2
    assert 30 < sr["ideal_ms"] < 50


@pytest.mark.parametrize("a_t,b_t,mode", [(False, False, "1"), (True, False, "1"), (False, True, "a"),
                                          (True, True, "b"), (False, False, "0")])
def test_gemm_variants_compile_for_sm100a(pkg, cg, monkeypatch, a_t, b_t, mode):
    """Every tensor-core GEMM variant compiles with NVRTC for sm_100a (no device needed): operands
    K-major or MN-major, split in the kernel or by a pass, with a last-wave split, with split-K, with
    and without the TMA-store epilogue."""
    import importlib
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    ir = importlib.import_module("tensor-compiler-webgpu_b200.ir")
    monkeypatch.setenv("TCB_GEMM_FUSED", mode)
    for Bt, M, K, N in ((150, 128, 256, 64), (1, 256, 4096, 128), (2, 300, 96, 130)):
        g = ir.Graph()
        x = g.input("x", [Bt, K, M] if a_t else [Bt, M, K])
        y = g.input("y", [Bt, N, K] if b_t else [Bt, K, N])
        a = g.transpose(x, [0, 2, 1]) if a_t else x
        b = g.transpose(y, [0, 2, 1]) if b_t else y
        out = g.tanh(g.matmul(a, b))
        f = pkg.fuse.fuse(g, keep=[out])
        for lau in cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=[f.index[out]])["launches"]:
            assert rt.compile_check(lau.code) > 0


def test_multi_instance_modules_compile(cg):
    import importlib
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    for src in (cg.copy_source(4), cg.copy_source(1), cg.split_multi_source()):
        assert rt.compile_check(src) > 0


def test_plain_launch_cache_follows_the_gemm_overrides(pkg, monkeypatch):
    """A one-op matmul lowered under one GEMM override is not reused under another: the cache is keyed by
    the overrides too (a reference lowering under TCB_GEMM_FUSED=0 must split its operands by passes even
    after a default lowering of the same shapes)."""
    import importlib
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    g = pkg.ir.Graph()
    g.matmul(g.input("a", [64, 128]), g.input("b", [128, 64]))
    monkeypatch.delenv("TCB_GEMM_FUSED", raising=False)
    (a,) = cg.lower(g, matmul="tiled")["launches"]
    monkeypatch.setenv("TCB_GEMM_FUSED", "0")
    (b,) = cg.lower(g, matmul="tiled")["launches"]
    assert a.info["fused_split"] == (True, True) and b.info["fused_split"] == (False, False)


def test_transposed_products(cg):
    """A plain tensor-core matmul read only by a transposeLast2 becomes one GEMM computing the transposed
    product (B^T.A^T, operands through their folds, the mixed 3xTF32 terms in the untransposed order);
    not when the matmul is kept or read elsewhere, when the transpose itself folds into a GEMM, or on the
    CUDA-core path."""
    import importlib
    ir = importlib.import_module("tensor-compiler-webgpu_b200.ir")
    g = ir.Graph()
    a = g.input("a", [4, 64, 256])
    b = g.input("b", [4, 256, 256])
    m = g.matmul(a, b)                          # [4, 64, 256], read only by t
    t = g.transpose(m, [0, 2, 1])               # [4, 256, 64]
    out = g.relu(t)
    m2 = g.matmul(a, b)
    t2 = g.transpose(m2, [0, 2, 1])
    shared = g.exp(m2)                          # m2 has another reader: no rewrite
    m3 = g.matmul(a, b)
    t3 = g.transpose(m3, [0, 2, 1])
    w = g.input("w", [4, 64, 32])
    prod = g.matmul(t3, w)                      # t3 folds into this GEMM's operand instead
    keep = [out, t2, shared, prod]
    low = cg.lower_fused(g, matmul="tiled", fold=True, keep=keep)
    assert low["transposed"] == [(t, m)]
    lau = next(l for l in low["launches"] if l.node == t)
    assert lau.inputs == [b, a] and lau.info["mnk"] == (4, 256, 256, 64)
    assert (lau.info["a_t"], lau.info["b_t"]) == (True, True)
    assert "#define TCB_CROSS_BA 1" in lau.code
    assert m not in {l.node for l in low["launches"]}
    assert cg.lower_fused(g, matmul="tiled", fold=True, keep=keep + [m])["transposed"] == []
    assert cg.lower_fused(g, matmul="naive", fold=True, keep=keep)["transposed"] == []
    assert cg.lower_fused(g, matmul="tiled", keep=keep)["transposed"] == []


def test_c5_attention_products_transposed(pkg, cg):
    import importlib
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    cfg, c = wl.c5_cfg(batch=64)
    gs = pkg.steps.build_grad3b(c["V"], 64, cfg)
    k0 = [gs["loss"], *gs["grads"].values()]
    f = pkg.fuse.fuse(gs["graph"], keep=k0)
    keep = [f.index[i] for i in k0]
    low = cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep, colfuse=True, mofuse=True)
    tl = {t: m for t, m in low["transposed"]}
    assert len(tl) == cfg["L"]
    for l in low["launches"]:
        if l.node in tl:
            assert l.info["mnk"][1:] == (256, 256, 64) and l.info["bn"] == 64
