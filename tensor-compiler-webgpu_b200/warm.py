"""Fill the on-disk kernel cache for the standard workloads (NVRTC, no GPU needed).

Every fused node is its own NVRTC instantiation, so a cold process spends
seconds compiling; build() runs this once so the benches, tests and smoke
load cubins instead.  The cache is keyed by a hash of each kernel's full
source, so a changed template or body simply misses.
"""
from __future__ import annotations

from . import codegen as cg
from . import runtime as rt
from . import workloads as wl
from .fuse import fuse
from . import steps as _steps
from .cases import fused_direct_cases


def _codes(graph, keep=(), matmul="naive"):
    """Kernels of a graph fused (as verified, and as a resident program with column sums in their
    producers) and unfused."""
    f = fuse(graph, keep=list(keep))
    fk = [f.index[k] for k in keep]
    return {lau.code for lau in cg.lower_fused(f.graph, matmul=matmul)["launches"]} | \
        {lau.code for lau in cg.lower_fused(f.graph, matmul=matmul, colfuse=True, keep=fk)["launches"]} | \
        {lau.code for lau in cg.lower_fused(f.graph, matmul=matmul, colfuse=True, mofuse=True, keep=fk)["launches"]} | \
        {lau.code for lau in cg.lower(graph, matmul=matmul)["launches"]}


def standard_sources(full=True):
    codes = set()
    for c in fused_direct_cases():
        codes |= _codes(c["graph"], matmul=c.get("matmul", "naive"))
    W = wl.c2_graph(256, 1024)
    codes |= _codes(W["graph"], W["keep"])
    for R, C in ((64, 8192), (257, 1000)):
        W = wl.c2_graph(R, C)
        codes |= _codes(W["graph"], W["keep"])
    for what in ("softmax", "logsoftmax", "rowsum"):
        for R, C in ((300, 4096), (64, 10), (5, 4097)):
            W = wl.c4_graph(R, C, what)
            codes |= _codes(W["graph"], W["keep"])
    for M, K, N in ((256, 4096, 128), (130, 1024, 96)):
        for act in ("relu", "tanh"):
            W = wl.c3_graph(M, K, N, act)
            codes |= _codes(W["graph"], W["keep"], "naive") | _codes(W["graph"], W["keep"], "tiled")
    step = wl.c1_step(64)
    codes |= _codes(step["graph"], [step["loss"], *step["outputs"].values()])
    if full:
        W = wl.c2_graph(8192, 8192)
        codes |= _codes(W["graph"], W["keep"])
        W = wl.c4_graph(65536, 4096, "softmax")
        codes |= _codes(W["graph"], W["keep"])
        W = wl.c3_graph(4096, 4096, 4096, "relu")
        codes |= _codes(W["graph"], W["keep"], "tiled")
        cfg, c = wl.c5_cfg()
        gs = _steps.build_grad3b(c["V"], c["batch"], cfg)
        f = fuse(gs["graph"], keep=[gs["loss"], *gs["grads"].values()])
        keep = [f.index[i] for i in [gs["loss"], *gs["grads"].values()]]
        codes |= {lau.code for lau in cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep)["launches"]}
        codes |= {lau.code for lau in cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep,
                                                     colfuse=True)["launches"]}
        codes |= {lau.code for lau in cg.lower_fused(f.graph, matmul="tiled", fold=True, keep=keep,
                                                     colfuse=True, mofuse=True)["launches"]}
        ad = _steps.build_adam_graph(c["V"], cfg)
        fa = fuse(ad["graph"], keep=list(ad["outputs"].values()))
        codes |= {lau.code for lau in cg.lower_fused(fa.graph, matmul="tiled")["launches"]}
    return codes


def sweep_sources():
    from . import timing as tm
    codes = set()
    for w in tm.workloads():
        for p in tm.build_variants(w)["programs"].values():
            codes |= {d["code"] for d in p["dispatches"]}
    return codes | {c["program"]["dispatches"][0]["code"] for c in tm.ceiling_programs()}


def fuzz_sources(every=10):
    """Kernels of the differential fuzzer's runs over corpus programs i % every in {1, 2}."""
    from .autodiff import grad
    from .corpus import corpus_program
    codes = set()
    for i in range(1, 2001):
        if every != 1 and i % every not in (1, 2):
            continue
        p = corpus_program(i, f32=True)
        G = grad(p.graph, p.outputs, [n.id for n in p.graph.inputs()])
        mms = ("naive", "tiled") if any(n.op == "matmul" for n in p.graph.nodes) else ("naive",)
        for mm in mms:
            for g, keep in ((p.graph, p.outputs), (G.graph, list(p.outputs) + list(G.grads))):
                codes |= _codes(g, keep, mm)
    return codes


def full_size_sources():
    """Kernels of the BASELINE configs at full size (C2, C3 both shapes with relu and tanh, C4 softmax,
    logSoftmax and row sum) and of the value sabotages over the direct cases."""
    codes = set()
    W = wl.c2_graph(8192, 8192)
    codes |= _codes(W["graph"], W["keep"])
    for M, K, N in wl.C3_SHAPES:
        for act in ("relu", "tanh"):
            W = wl.c3_graph(M, K, N, act)
            codes |= _codes(W["graph"], W["keep"], "tiled")
    for what in ("softmax", "logsoftmax", "rowsum"):
        W = wl.c4_graph(65536, 4096, what)
        codes |= _codes(W["graph"], W["keep"])
    for c in fused_direct_cases():
        f = fuse(c["graph"])
        for s in ("epilogue-before-bias", "layernorm-tree-short", "softmax-no-max"):
            codes |= {lau.code for lau in cg.lower_fused(f.graph, matmul=c.get("matmul", "naive"),
                                                         sabotage=s)["launches"]}
    return codes


def graph_sources(graphs):
    """Kernels of (graph, keep) pairs on both matmul paths, fused and unfused."""
    codes = set()
    for g, keep in graphs:
        for mm in ("naive", "tiled"):
            codes |= _codes(g, keep, mm)
    return codes


def warm(full=True, prune=True, extra=()):
    """Compile the standard kernels (and the sources in `extra`) into the cache; with `prune`, drop
    cached cubins of other sources (old templates or codegen) so the cache that travels with the tree
    stays small."""
    import os
    codes = standard_sources(full) | set(extra)
    if full:
        codes |= sweep_sources() | fuzz_sources(10) | full_size_sources()
    n = rt.precompile(codes)
    if prune and full and os.path.isdir(rt.CACHE_DIR):
        keep = {os.path.basename(rt._cache_path(c)) for c in codes}
        for name in os.listdir(rt.CACHE_DIR):
            if name.endswith(".cubin") and name not in keep:
                os.unlink(os.path.join(rt.CACHE_DIR, name))
    return n
