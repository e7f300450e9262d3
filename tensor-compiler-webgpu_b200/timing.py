"""The timing harness and the fusion sweep: the replacement of src/fusion/bench.js and
src/fusion/workloads.js on the B200.

* ``Bench`` (bench.js:19-216): ``create``, ``info``, ``pipeline``, ``prepare(program)``,
  ``reset``, ``outputs``, ``rep(prepared, k)``, ``time(prepared_by_variant)``, ``destroy``, and the
  counters that check nothing is allocated or compiled inside a timed region (bench.js:41-47,
  201-208).  A repetition is k back-to-back runs of a program between two CUDA events on the
  launching stream (the reference's timestamp queries around one compute pass); wall time is taken
  beside it.  The protocol is amendment 32's: k so a repetition is >= 2 ms (at most 4096), 5 warm-up
  repetitions per variant, 32 repetitions per variant in ABBA order, median / min / max.
* Programs (workloads.js:155-175): ``{buffers: [{bytes, data}], dispatches: [{code, calls,
  bindings, scratch, label}], outputs, bytes, launches}``; ``graph_program`` counts bytes by
  amendment 33 (each distinct operand once at its own size, plus the output).
* ``workloads()`` / ``build_variants`` (workloads.js:76-126, 249-265): the amendment-34 sweep --
  unary and binary chains, matmul epilogues (naive: CUDA cores; tiled: tcgen05 3xTF32), LayerNorm
  and softmax rows, broadcast-recompute, lost reuse, the model's forward and step -- as unfused,
  fused, recompute and matmul-only variants.  The third-party hand-written kernels of the reference's
  sweep are not part of this backend.
* ``gate`` (web/m4-bench.html:116-146): before a workload is timed, each variant runs once and its
  outputs are judged against the float64 reference (a judge the caller supplies); a variant that fails
  is not timed.
* ``ceiling_programs`` (workloads.js:305-345): pure-read and copy kernels over 128 MiB, 32/64/128-bit
  elements, 256 / 1024 / 4096 CTAs of 256 threads, grid-strided: the measured HBM ceiling.
"""
from __future__ import annotations

import math
import time

import numpy as np

from . import runtime as rt
from .codegen import lower, lower_fused, KernelCall
from .fuse import fuse
from .ir import Graph, size
from .rng import Rng
from .cases import layer_norm_graph, unary_chain
from .steps import gelu, build_forward, build_step3b, init_params, param_shapes, adam_initial_state

WARMUP = 5
REPS = 32
TARGET_NS = 2e6
MAX_K = 4096


def median(a):
    s = sorted(a)
    n = len(s)
    return s[(n - 1) // 2] if n % 2 else (s[n // 2 - 1] + s[n // 2]) / 2


def summarize(reps):
    """median / min / max of per-run GPU ns and wall ms (bench.js:211-216)."""
    g = [r["gpuNs"] for r in reps]
    w = [r["wallMs"] for r in reps]
    return {"gpuNs": {"median": median(g), "min": min(g), "max": max(g)},
            "wallMs": {"median": median(w), "min": min(w), "max": max(w)}, "n": len(reps)}


class Bench:
    """bench.js's Bench over libtcb200 (one device, its stream, CUDA events)."""

    @staticmethod
    def create(device=0):
        return Bench(rt.GpuRunner.create(device))

    def __init__(self, runner):
        self.runner = runner
        self.counts = {}
        self.events = rt.Events(runner, 2)

    def _count(self, name):
        self.counts[name] = self.counts.get(name, 0) + 1

    def info(self):
        return {**self.runner.info(), "timestamps": "cuda events"}

    def pipeline(self, code):
        if code not in self.runner.pipelines:
            self._count("compile")
        return self.runner.pipeline(code)

    def prepare(self, program):
        bufs = []
        for b in program["buffers"]:
            self._count("alloc")
            buf = rt.DeviceBuffer(self.runner, max(16, b["bytes"]))
            if b.get("data") is not None:
                buf.upload(np.asarray(b["data"], dtype=np.float32).reshape(-1))
            bufs.append(buf)
        scratch_bytes = max([d.get("scratch", 0) for d in program["dispatches"]] + [0])
        scratch = None
        if scratch_bytes:
            self._count("alloc")
            scratch = rt.DeviceBuffer(self.runner, scratch_bytes)
            rt.check(rt.lib().tc_memset32(self.runner.ctx, scratch.ptr, 0, scratch_bytes // 4))
        h = rt.ctypes.c_void_p()
        rt.check(rt.lib().tc_plan_create(self.runner.ctx, rt.ctypes.byref(h)))
        for d in program["dispatches"]:
            mod = self.pipeline(d["code"])
            ptrs = [bufs[i].ptr for i in d["bindings"]]
            for call in d["calls"]:
                rt.issue(call, mod, ptrs[:-1], ptrs[-1], scratch.ptr if scratch else 0, plan=h)
        return {"program": program, "buffers": bufs, "scratch": scratch, "plan": h}

    def reset(self, prepared):
        for b, buf in zip(prepared["program"]["buffers"], prepared["buffers"]):
            if b.get("data") is not None:
                buf.upload(np.asarray(b["data"], dtype=np.float32).reshape(-1))

    def outputs(self, prepared):
        rt.check(rt.lib().tc_plan_run(prepared["plan"]))
        self.runner.sync()
        prog = prepared["program"]
        return [prepared["buffers"][i].download(prog["buffers"][i]["bytes"] // 4) for i in prog["outputs"]]

    def rep(self, prepared, k):
        """One timed repetition: k runs of the program between two events on the launching stream."""
        ev = self.events
        t0 = time.perf_counter()
        ev.record(0)
        for _ in range(k):
            rt.check(rt.lib().tc_plan_run(prepared["plan"]))
        ev.record(1)
        self.runner.sync()
        wall = (time.perf_counter() - t0) * 1e3
        return {"gpuNs": ev.ms(0, 1) * 1e6, "wallMs": wall}

    def snapshot(self):
        return dict(self.counts)

    @staticmethod
    def created(before, after):
        return {k: after.get(k, 0) - before.get(k, 0) for k in set(before) | set(after)
                if after.get(k, 0) != before.get(k, 0)}

    def time(self, prepared):
        """Amendment 32's protocol over the variants of one workload (bench.js:175-195)."""
        names = list(prepared)
        self.rep(prepared[names[0]], 1)
        first = self.rep(prepared[names[0]], 1)
        k = max(1, min(MAX_K, math.ceil(TARGET_NS / max(first["gpuNs"], 1))))
        for n in names:
            for _ in range(WARMUP):
                self.rep(prepared[n], k)
        reps = {n: [] for n in names}
        before = self.snapshot()
        for b in range(REPS):
            order = names if b % 2 == 0 else names[::-1]
            for n in order:
                r = self.rep(prepared[n], k)
                reps[n].append({"gpuNs": r["gpuNs"] / k, "wallMs": r["wallMs"] / k})
        return {"k": k, "reps": reps, "created": Bench.created(before, self.snapshot())}

    def destroy(self, prepared):
        rt.check(rt.lib().tc_plan_free(prepared["plan"]))
        for b in prepared["buffers"]:
            b.free()
        if prepared["scratch"]:
            prepared["scratch"].free()

    def close(self):
        self.events.free()
        self.runner.close()


# ---------------------------------------------------------------- programs
def graph_program(graph, lowered, inputs, outputs):
    """A lowered graph as a program: a buffer per node, bytes by amendment 33 (workloads.js:155-175)."""
    buffers = []
    for n in graph.nodes:
        count = max(1, size(n.shape))
        data = None
        if n.op == "input":
            data = np.asarray(inputs[n.attrs["name"]], dtype=np.float32)
        elif n.op == "const":
            v = n.attrs["value"]
            data = np.full(count, v, np.float32) if isinstance(v, (int, float)) else np.asarray(v, np.float32)
        buffers.append({"bytes": count * 4, "data": data})
    dispatches = []
    nbytes = 0
    for lau in lowered["launches"]:
        dispatches.append({"code": lau.code, "calls": lau.calls, "bindings": [*lau.inputs, lau.node],
                           "scratch": lau.scratch_bytes, "label": lau.pattern or lau.kind})
        nbytes += lau.bytes
    return {"buffers": buffers, "dispatches": dispatches, "outputs": list(outputs), "bytes": nbytes,
            "launches": len(dispatches)}


CHAIN_LENGTHS = (1, 2, 4, 8, 16)
CHAIN_SIZES = (1000, 65537, 1048573, 4194301)
BINARY_LENGTHS = (1, 2, 4, 8)
BINARY_SIZES = (65537, 4194301)
MATMUL_SHAPES = ((512, 64, 64), (512, 64, 256), (512, 256, 64), (1000, 63, 257), (4096, 64, 256), (128, 1024, 128),
                 (2048, 512, 512))
ROW_C = (1, 7, 64, 65, 256, 1000, 4096)
ROW_R = (1, 64, 4096, 65536)
ROW_CAP = 2 ** 22
BROADCAST_R = (16, 256, 4096)
REUSE_SIZE = 1048573


def _draw_inputs(graph, seed, ranges=None):
    rng = Rng(seed)
    out = {}
    for n in graph.inputs():
        lo, hi = (ranges or {}).get(n.attrs["name"], (-2, 2))
        out[n.attrs["name"]] = rng.uniform_array(size(n.shape), lo, hi).astype(np.float32)
    return out


def _graph_workload(wid, family, params, build, variants=("unfused", "fused"), matmul="naive", ranges=None, seed=1):
    def make():
        g = Graph()
        outs = build(g)
        outs = list(outs) if isinstance(outs, (list, tuple)) else [outs]
        return g, outs, _draw_inputs(g, seed, ranges)
    return {"id": wid, "family": family, "params": params, "variants": list(variants), "matmul": matmul, "make": make,
            "judge": "composed"}


def _binary_chain(g, n, L):
    y = g.input("x0", [n])
    ops = ("add", "mul", "sub")
    for k in range(1, L + 1):
        y = getattr(g, ops[(k - 1) % 3])(y, g.input(f"x{k}", [n]))
    return y


def workloads():
    """Every workload of the amendment-34 sweep, in timing order (workloads.js:76-126), minus the
    third-party hand-written baselines."""
    w = []
    for n in CHAIN_SIZES:
        for L in CHAIN_LENGTHS:
            w.append(_graph_workload(f"chain-unary-L{L}-n{n}", "chain-unary", {"L": L, "n": n},
                                     lambda g, n=n, L=L: unary_chain(g, g.input("x", [n]), L)))
    for n in BINARY_SIZES:
        for L in BINARY_LENGTHS:
            w.append(_graph_workload(f"chain-binary-L{L}-n{n}", "chain-binary", {"L": L, "n": n},
                                     lambda g, n=n, L=L: _binary_chain(g, n, L)))
    for matmul in ("naive", "tiled"):
        for M, K, N in MATMUL_SHAPES:
            for act in ("relu", "gelu"):
                def build(g, M=M, K=K, N=N, act=act):
                    y = g.add(g.matmul(g.input("a", [M, K]), g.input("w", [K, N])), g.input("bias", [N]))
                    return g.relu(y) if act == "relu" else gelu(g, y)
                w.append(_graph_workload(f"matmul-{matmul}-{act}-{M}x{K}x{N}", "matmul-epilogue",
                                         {"M": M, "K": K, "N": N, "act": act, "matmul": matmul}, build, matmul=matmul,
                                         ranges={"w": (-1 / math.sqrt(K), 1 / math.sqrt(K))}))
    for pattern in ("layernorm", "softmax"):
        for C in ROW_C:
            for R in ROW_R:
                if R * C > ROW_CAP or C == 1:
                    continue
                if pattern == "layernorm":
                    build = (lambda g, R=R, C=C: layer_norm_graph(g, g.input("x", [R, C]), g.input("g", [C]),
                                                                  g.input("b", [C])))
                else:
                    build = lambda g, R=R, C=C: g.softmax(g.input("x", [R, C]), 1)
                w.append(_graph_workload(f"{pattern}-R{R}-C{C}", pattern, {"R": R, "C": C}, build))
    for R in BROADCAST_R:
        w.append(_graph_workload(f"broadcast-recompute-R{R}", "broadcast-recompute", {"R": R, "C": 256, "ops": 16},
                                 lambda g, R=R: g.add(g.input("y", [R, 256]), unary_chain(g, g.input("p", [256]), 16)),
                                 variants=("unfused", "fused", "recompute")))
    for ops in (1, 16):
        def lost(g, ops=ops):
            t = unary_chain(g, g.input("x", [REUSE_SIZE]), ops)
            return [g.mul(t, g.const(2)), g.add(t, g.const(1)), g.tanh(t), g.exp(g.neg(t))]
        w.append(_graph_workload(f"lost-reuse-{ops}op", "lost-reuse", {"ops": ops, "consumers": 4, "n": REUSE_SIZE},
                                 lost, variants=("unfused", "fused", "recompute")))
    for V, B in ((16, 8), (75, 16)):
        w.append(_model_workload("forward", V, B))
    for V, B in ((16, 8), (16, 16), (75, 16)):
        w.append(_model_workload("step", V, B))
    return w


def _model_workload(what, V, B):
    def make():
        rng = Rng(V * 1000 + B)
        toks = [rng.int(0, V - 1) for _ in range(B * 64)]
        targets = [rng.int(0, V - 1) for _ in range(B * 64)]

        def onehot(ids):
            a = np.zeros(len(ids) * V, np.float32)
            a[np.arange(len(ids)) * V + np.asarray(ids)] = 1
            return a
        params = {k: np.asarray(v, np.float32) for k, v in init_params(V, 1).items()}
        if what == "forward":
            f = build_forward(V, B)
            return f["graph"], [f["logits"], f["loss"]], {**params, "x": onehot(toks), "y": onehot(targets)}
        st = build_step3b(V, B)
        state = adam_initial_state(st["names"], param_shapes(V))
        return st["graph"], [st["loss"], *st["outputs"].values()], {**params, **state, "x": onehot(toks),
                                                                    "y": onehot(targets), st["cotangent"]: [1.0]}
    variants = ("unfused", "fused", "matmul-only") if what == "step" else ("unfused", "fused")
    return {"id": f"{what}-V{V}-B{B}", "family": "training-step" if what == "step" else "forward",
            "params": {"V": V, "B": B}, "variants": list(variants), "matmul": "naive", "make": make,
            "judge": "compare"}


def build_variants(w):
    """Every variant of a workload as a program (workloads.js:249-265)."""
    graph, outputs, inputs = w["make"]()
    programs = {}
    for v in w["variants"]:
        if v in ("unfused", "matmul-only"):
            low = lower(graph, matmul=w["matmul"])
            if v == "matmul-only":
                low = {"launches": [l for l in low["launches"] if l.op == "matmul"]}
            programs[v] = graph_program(graph, low, inputs, outputs)
        else:
            f = fuse(graph, keep=outputs, recompute=(v == "recompute"))
            p = graph_program(f.graph, lower_fused(f.graph, matmul=w["matmul"]), inputs,
                              [f.index[o] for o in outputs])
            p["fusedNodes"] = sum(1 for n in f.graph.nodes if n.op == "fused")
            programs[v] = p
    return {"graph": graph, "outputs": outputs, "inputs": inputs, "programs": programs}


# ---------------------------------------------------------------- the bandwidth ceiling
CEILING_BYTES = 128 * 2 ** 20
_WIDTH = {"u32": ("unsigned int", 1), "vec2": ("uint2", 2), "vec4": ("uint4", 4)}


def _ceiling_source(mode, width):
    T, lanes = _WIDTH[width]
    fold = {"u32": "acc", "vec2": "acc.x ^ acc.y", "vec4": "acc.x ^ acc.y ^ acc.z ^ acc.w"}[width]
    xor = {"u32": "acc ^= v;", "vec2": "acc.x ^= v.x; acc.y ^= v.y;",
           "vec4": "acc.x ^= v.x; acc.y ^= v.y; acc.z ^= v.z; acc.w ^= v.w;"}[width]
    zero = "0u" if width == "u32" else f"make_{T}(" + ", ".join(["0u"] * lanes) + ")"
    if mode == "read":
        body = f"""  {T} acc = {zero};
  for (u64 i = g; i < n; i += stride) {{ const {T} v = src[i]; {xor} }}
  reinterpret_cast<unsigned int*>(a.out)[g] = {fold};"""
    else:
        body = "  for (u64 i = g; i < n; i += stride) dst[i] = src[i];"
    return f"""// {mode} ceiling, {width}
#include "tcb/common.cuh"
extern "C" __global__ void __launch_bounds__(256) tcb_ceiling(const tcb::Args a) {{
  tcb::grid_dependency_sync();
  const {T}* __restrict__ src = reinterpret_cast<const {T}*>(a.in[0]);
  {T}* __restrict__ dst = reinterpret_cast<{T}*>(a.out);
  (void)dst;
  const u64 n = (u64)a.p[0];
  const u64 g = (u64)blockIdx.x * blockDim.x + threadIdx.x;
  const u64 stride = (u64)gridDim.x * blockDim.x;
{body}
}}
"""


def ceiling_programs():
    """Pure-read and copy over 128 MiB: 32/64/128-bit elements x 256/1024/4096 CTAs of 256 (workloads.js:312-345)."""
    out = []
    for mode in ("read", "copy"):
        for width in ("u32", "vec2", "vec4"):
            for groups in (256, 1024, 4096):
                lanes = _WIDTH[width][1]
                n = CEILING_BYTES // (4 * lanes)
                call = KernelCall("tcb_ceiling", (groups, 1, 1), (256, 1, 1), 0, [n])
                dst_bytes = groups * 256 * 4 if mode == "read" else CEILING_BYTES
                prog = {"buffers": [{"bytes": CEILING_BYTES, "data": None}, {"bytes": dst_bytes, "data": None}],
                        "dispatches": [{"code": _ceiling_source(mode, width), "calls": [call], "bindings": [0, 1],
                                        "scratch": 0, "label": f"{mode} {width}"}],
                        "outputs": [], "bytes": CEILING_BYTES if mode == "read" else 2 * CEILING_BYTES,
                        "launches": 1}
                out.append({"id": f"{mode}-{width}-x{groups}", "mode": mode, "width": width, "groups": groups,
                            "program": prog})
    return out


def compare_outputs(a, b):
    """The model workloads' gate (workloads.js:370-374): the largest difference between two variants'
    outputs, and whether all are finite."""
    diffs = [float(np.max(np.abs(x.astype(np.float64) - y))) if x.size else 0.0 for x, y in zip(a, b)]
    finite = all(np.isfinite(x).all() for x in a) and all(np.isfinite(x).all() for x in b)
    return {"finite": bool(finite), "maxAbs": max(diffs) if diffs else 0.0, "lossDiff": diffs[0] if diffs else 0.0}


def gate(bench, w, v, prepared, judge):
    """Each variant once, its outputs judged before anything is timed (web/m4-bench.html:116-146).

    `judge(graph, inputs, outputs, gpu_outputs) -> {"pass", ...}` judges one variant's outputs against
    the float64 reference with amendment 8's composed bound (workloads.js:275-301 streamingReference,
    :351-367 judgeOutputs); the caller supplies it (the checker is test infrastructure, not part of this
    package).  The model workloads, whose composed bound is vacuous, compare fused with unfused instead."""
    outs = {name: bench.outputs(p) for name, p in prepared.items() if name != "matmul-only"}
    g = {}
    if w.get("judge", "composed") == "composed":
        for name, o in outs.items():
            j = judge(v["graph"], v["inputs"], v["outputs"], o)
            g[name] = {k: j.get(k) for k in ("pass", "unjudged", "worst", "unjudgeable", "elements", "first")}
    else:
        c = compare_outputs(outs["fused"], outs["unfused"])
        g["fusedVsUnfused"] = c
        g["fused"] = {"pass": c["finite"]}
        g["unfused"] = {"pass": all(np.isfinite(x).all() for x in outs["unfused"])}
    failed = [k for k, r in g.items() if r.get("pass") is False]
    return {"pass": not failed, "failed": failed, "variants": g}


def run_sweep(bench, only=None, families=None, log=None, judge=None):
    """Time every workload's variants and the ceiling programs; returns a list of result records.

    Every workload is gated first (`gate`): a variant whose outputs fail the judge is not timed."""
    if judge is None:
        raise ValueError("run_sweep needs a judge: every variant's outputs are checked before it is timed")
    results = []
    for c in ceiling_programs():
        if only and not any(s in c["id"] for s in only):
            continue
        p = bench.prepare(c["program"])
        t = bench.time({"ceiling": p})
        s = summarize(t["reps"]["ceiling"])
        results.append({"id": c["id"], "family": "ceiling", "k": t["k"], "created": t["created"],
                        "GBps": c["program"]["bytes"] / s["gpuNs"]["median"], **s})
        bench.destroy(p)
        if log:
            log(results[-1])
    for w in workloads():
        if only and not any(s in w["id"] for s in only):
            continue
        if families and w["family"] not in families:
            continue
        v = build_variants(w)
        prepared = {name: bench.prepare(p) for name, p in v["programs"].items()}
        gt = gate(bench, w, v, prepared, judge)
        if not gt["pass"]:
            results.append({"id": w["id"], "family": w["family"], "params": w["params"], "gate": gt,
                            "failedGate": gt["failed"], "created": {}, "variants": {}})
            for p in prepared.values():
                bench.destroy(p)
            if log:
                log(results[-1])
            continue
        for p in prepared.values():
            bench.reset(p)
        t = bench.time(prepared)
        rec = {"id": w["id"], "family": w["family"], "params": w["params"], "k": t["k"], "created": t["created"],
               "gate": gt, "variants": {}}
        for name, p in v["programs"].items():
            s = summarize(t["reps"][name])
            rec["variants"][name] = {"launches": p["launches"], "bytes": p["bytes"],
                                     "GBps": p["bytes"] / s["gpuNs"]["median"], **s}
        for p in prepared.values():
            bench.destroy(p)
        results.append(rec)
        if log:
            log(rec)
    return results
