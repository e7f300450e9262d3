"""bench.py -- the driver's benchmark contract for the fused-kernel hot path.

One JSON line.  Its headline (`value`) is BASELINE.json configs[1] (C2): the fused elementwise chain on
fp32 [8192, 8192], forward + autodiff backward, as the fused launch list the fusion pass gives.  A step =
every launch of that list once, inputs resident in HBM (each operand is 256 MiB, twice the 126 MB L2, so
no flush is needed between steps).  value = algorithmic bytes per step / device time, summed over ranks,
the bytes counted over the reference fused plan's launches (amendment 33: each distinct operand once at
its own size, plus the output) -- the same unit the reference arm counts.  The resident program moves
fewer bytes than that plan (column sums and elementwise readers run in their producers' passes, unread
launches are left out); `config.moved_gbs` is the bandwidth of the bytes it does move.

The rest of the metric rides in `records`, each with its own roofline, clocks, end-to-end figure and
(rank 0, one GPU) CPU baseline:
  c1 -- the MLP step (samples/s, launch-bound, one CUDA graph);
  c3 -- the matmul + bias + relu/tanh on the tcgen05 3xTF32 path, both BASELINE shapes (TFLOP/s);
  c4 -- softmax and logSoftmax forward + backward on [65536, 4096], 1 % of rows +800 (GB/s);
  train -- the C5 decoder transformer's training step (tokens/s), data parallel over every rank:
           each rank runs its shard of the global batch 512; the gradients are sum-allreduced over NCCL
           (the library's own communicator) in buckets on a collective stream during the backward,
           and every rank runs the same Adam program.
With --gpus N (one process per GPU, torchrun), C2 runs as N replicas (no data-path collective, `scaling`
weak) and `train` runs the global batch over the N ranks (strong scaling); c1/c3/c4 are 1-GPU records.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload all|c1|c2|c3|c4|c5]
  python bench.py --impl reference ...   (the reference's CPU path: the C restatement of interp.js)
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = "tensor-compiler-webgpu_b200"
METRIC = "fused-kernel HBM GB/s (% peak); train tokens/s at 1/2/4/8 B200 vs f64 interp"
FALLBACK_HBM = 6650.0


def _mods():
    pkg = importlib.import_module(PKG)
    return (pkg, importlib.import_module(PKG + ".runtime"), importlib.import_module(PKG + ".codegen"),
            importlib.import_module(PKG + ".workloads"))


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region (reads only)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = os.path.join("/tmp", f"tcb_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _init_group(world):
    """torch.distributed carries only host plumbing here (barriers, the max over ranks, the NCCL unique
    id): a gloo group with a short timeout.  The data-path collective is the library's own NCCL."""
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))


def _max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _sm_mhz_of_peak():
    """The median SM clock under which MEASURED_PEAKS.json's bf16 burst was sampled (None if unknown)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["clocks_under_load"]["sm_mhz_median"])
    except Exception:
        return None


C3_DEFAULT = (4096, 4096, 4096)


def build_workload(name, wl, pkg, cg, rows=None, variant=None, shape=None):
    """(graph, fused, lowered, inputs, keep, config, W) for a graph workload at its BASELINE size
    (`rows` cuts C2/C4 to fewer rows: the small case a detailed ncu capture runs on; `variant` is C3's
    activation or C4's function, `shape` C3's (M, K, N))."""
    if name == "c2":
        W = wl.c2_graph(rows or 8192, 8192)
        inputs = wl.c2_inputs(W)
        cfg = {"workload": "C2 elementwise chain fp32 [8192,8192] fwd+bwd", "ops": W["ops"],
               "row_broadcast": "[1,8192]", "l2": "operands 256 MiB > 126 MB L2, no flush"}
    elif name == "c4":
        what = variant or "softmax"
        W = wl.c4_graph(rows or 65536, 4096, what)
        inputs, _ = wl.c4_inputs(W)
        cfg = {"workload": f"C4 {what} fp32 [65536,4096] fwd+bwd, 1% rows +800", "l2": "1 GiB operands > L2"}
    elif name == "c3":
        M, K, N = shape or C3_DEFAULT
        act = variant or "relu"
        W = wl.c3_graph(M, K, N, act)
        inputs = wl.c3_inputs(M, K, N)
        cfg = {"workload": f"C3 matmul [{M},{K}]x[{K},{N}] + bias + {act} (fp32 via 3xTF32)",
               "l2": f"{(M * K + K * N + M * N) * 4 >> 20} MiB operands > L2"}
    else:
        raise SystemExit(f"unknown workload {name}")
    graph = W["graph"]
    fused = pkg.fuse.fuse(graph, keep=W["keep"])
    # the resident program's lowering: column sums and elementwise readers run inside their producers
    lowered = cg.lower_fused(fused.graph, matmul="tiled" if name == "c3" else "naive", colfuse=True, mofuse=True,
                             keep=[fused.index[k] for k in W["keep"]])
    return graph, fused, lowered, inputs, W["keep"], cfg, W


def cpu_sample(name, wl, pkg, cg, rows, variant=None, shape=None):
    """The same workload cut to `rows` rows (rows are independent in C2 and C4; an output row of C3 needs
    one row of A): graph, inputs, units.  Units are the metric's: algorithmic bytes (C2, C4), useful flops
    (C3), samples (C1), tokens (C5: `rows` sequences of the full training step: forward, backward, Adam)."""
    if name == "c1":
        step = wl.c1_step(64)
        inputs = wl.c1_inputs(64)
        inputs[step["cotangent"]] = [1.0]
        return step["graph"], inputs, 64
    if name == "c5":
        cfg, c = wl.c5_cfg()
        st = pkg.steps.build_step3b(c["V"], rows, cfg)
        params = pkg.steps.init_params_normal(c["V"], 0, 0.02, cfg)
        state = pkg.steps.adam_initial_state(st["names"], pkg.steps.param_shapes(c["V"], cfg))
        x, y = wl.one_hot_batch(wl.c5_tokens(rows, cfg["T"], c["V"]), c["V"])
        return st["graph"], {**params, **state, "x": x, "y": y, st["cotangent"]: [1.0]}, rows * cfg["T"]
    if name == "c3":
        M, K, N = shape or C3_DEFAULT
        W = wl.c3_graph(rows, K, N, variant or "relu")
        return W["graph"], wl.c3_inputs(rows, K, N), 2 * rows * K * N
    if name == "c2":
        W = wl.c2_graph(rows, 8192)
        inputs = wl.c2_inputs(W)
    else:
        W = wl.c4_graph(rows, 4096, variant or "softmax")
        inputs, _ = wl.c4_inputs(W)
    fused = pkg.fuse.fuse(W["graph"], keep=W["keep"])
    nbytes = sum(l.bytes for l in cg.lower_fused(fused.graph)["launches"])
    return W["graph"], inputs, nbytes


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: the CPU baseline (the reference's algorithm), never the measured GPU path
    oracle.build()
    return oracle


_SAMPLES = {}


def _cpu_worker(job):
    """One worker's share of a reference-arm step: evaluate its row sample, return (units, seconds)."""
    name, rows, reps, variant, shape = job
    key = (name, rows, variant, shape)
    if key not in _SAMPLES:
        pkg, cg, wl = (importlib.import_module(PKG), importlib.import_module(PKG + ".codegen"),
                       importlib.import_module(PKG + ".workloads"))
        _SAMPLES[key] = (_oracle(), *cpu_sample(name, wl, pkg, cg, rows, variant, shape))
    oracle, graph, inputs, nbytes = _SAMPLES[key]
    t0 = time.perf_counter()
    for _ in range(reps):
        oracle.evaluate(graph, inputs, want=[])
    return nbytes * reps, time.perf_counter() - t0


class _Stream:
    """A second CUDA stream of the runner's context, with events recorded on it."""

    def __init__(self, rt, runner):
        import ctypes
        self.rt, self.runner = rt, runner
        h = ctypes.c_uint64()
        rt.check(rt.lib().tc_stream_create(runner.ctx, ctypes.byref(h)))
        self.h = h.value

    def free(self):
        self.rt.check(self.rt.lib().tc_stream_destroy(self.runner.ctx, self.h))


def copy_ceiling(rt, runner, h_in, h_out, reps=3):
    """The end-to-end ceiling of one step's host traffic on this box: the same bytes as a step's inputs
    copied host -> device from the same pinned buffers while the same bytes as its outputs copy device ->
    host into the same pinned buffers, on two streams at once (plus each direction alone)."""
    lib = rt.lib()
    n_in = sum(h.nbytes for h in h_in)
    n_out = sum(h.nbytes for h in h_out)
    d_in = rt.DeviceBuffer(runner, max(n_in, 4))
    d_out = rt.DeviceBuffer(runner, max(n_out, 4))
    s1, s2 = _Stream(rt, runner), _Stream(rt, runner)
    ev = rt.Events(runner, 7)

    def rec(k, st):
        rt.check(lib.tc_event_record_on(runner.ctx, ev.ev[k], st))

    def h2d(st):
        off = 0
        for h in h_in:
            rt.check(lib.tc_memcpy_htod_on(runner.ctx, d_in.ptr + off, h.ptr, h.nbytes, st))
            off += h.nbytes

    def d2h(st):
        off = 0
        for h in h_out:
            rt.check(lib.tc_memcpy_dtoh_on(runner.ctx, h.ptr, d_out.ptr + off, h.nbytes, st))
            off += h.nbytes
    best = [math.inf, math.inf, math.inf]
    try:
        for _ in range(reps):
            rec(0, s1.h); h2d(s1.h); rec(1, s1.h)
            rt.check(lib.tc_event_sync(ev.ev[1], 60000))
            rec(2, s2.h); d2h(s2.h); rec(3, s2.h)
            rt.check(lib.tc_event_sync(ev.ev[3], 60000))
            rec(4, s1.h)                                               # both directions start together
            rt.check(lib.tc_stream_wait_event(runner.ctx, s2.h, ev.ev[4]))
            h2d(s1.h)
            d2h(s2.h)
            rec(6, s2.h)
            rt.check(lib.tc_stream_wait_event(runner.ctx, s1.h, ev.ev[6]))
            rec(5, s1.h)                                               # ... and end when both have
            rt.check(lib.tc_event_sync(ev.ev[5], 60000))
            best = [min(best[0], ev.ms(0, 1)), min(best[1], ev.ms(2, 3)), min(best[2], ev.ms(4, 5))]
    finally:
        runner.sync()
        ev.free()
        s1.free()
        s2.free()
        d_in.free()
        d_out.free()
    return {"h2d_gbs": round(n_in / best[0] / 1e6, 1) if n_in else None,
            "d2h_gbs": round(n_out / best[1] / 1e6, 1) if n_out else None,
            "both_ms": round(best[2], 3), "bytes": [n_in, n_out],
            "how": "one step's input bytes host->device and output bytes device->host from the same pinned "
                   "buffers, concurrently on two streams (best of 3)"}


def _timed(runner, rt, world, local, K, Wm, step, ev_pairs=0):
    """Warm up, then time exactly K calls of `step(k)` between a barrier + device sync on both sides,
    with the clocks sampled during the timed region; returns (total ms, events, clocks)."""
    ev = rt.Events(runner, 2 + 2 * ev_pairs)
    clocks = Clocks(local)   # sampled from the warm-up on: a short timed region may see no sample of its own
    clocks.start()
    time.sleep(0.3)
    for _ in range(Wm):
        step(None, ev)
    runner.sync()
    _barrier(world)
    ev.record(0)
    for k in range(K):
        step(k, ev)
    ev.record(1)
    runner.sync()
    clk = clocks.stop()
    _barrier(world)
    return ev.ms(0, 1), ev, clk


def graph_record(args, name, runner, world, rank, local, variant=None, shape=None, cpu=True):
    """One graph workload (C2, C3, C4) as a record: resident program, the dominant kernel timed live
    inside the timed region, end to end through the streaming API with its copy ceiling, CPU baseline."""
    pkg, rt, cg, wl = _mods()
    graph, fused, lowered, inputs, keep, cfg, W = build_workload(name, wl, pkg, cg, args.rows, variant, shape)
    if args.rows:
        cfg["workload"] += f" (cut to {args.rows} rows)"
    outs = [fused.index[k] for k in dict.fromkeys(keep)]
    prog = rt.Program(runner, fused.graph, lowered, keep=outs)
    launches = prog.launches   # the launches the step runs (a launch no output depends on is left out)
    moved_bytes = sum(l.bytes for l in launches)
    # the unit of work: the reference fused plan's algorithmic bytes (amendment 33 over the launches the
    # reference's lowerFused gives), as the reference arm and the CPU baseline count it; this program moves
    # fewer (column sums and readers in their producers' passes, unread launches left out)
    step_bytes = sum(l.bytes for l in cg.lower_fused(fused.graph, matmul="tiled" if name == "c3" else "naive")["launches"])
    name_of = {n.id: n.attrs["name"] for n in fused.graph.nodes if n.op == "input"}
    for nid, nm in name_of.items():
        prog.write(nid, inputs[nm])
    # the dominant kernel: the launch moving the most algorithmic bytes (C3: the tensor-core GEMM kernel)
    flat = [(k, c) for k, lau in enumerate(launches) for c in rt.program_calls(lau)]
    tensor = name == "c3"
    if tensor:
        dcall = next(i for i, (k, c) in enumerate(flat) if c.name in ("tcb_gemm_tc", "tcb_matmul"))
        dom = flat[dcall][0]
    else:
        dom = max(range(len(launches)), key=lambda k: launches[k].bytes)
        dcall = max(i for i, (k, c) in enumerate(flat) if k == dom)
    seg = rt.Segments(prog, [dcall, dcall + 1])
    K, Wm = args.steps, args.warmup

    def step(k, ev):
        seg.run(0)
        if k is not None:
            ev.record(2 + 2 * k)
        seg.run(1)
        if k is not None:
            ev.record(3 + 2 * k)
        seg.run(2)
    total_ms, ev, clk = _timed(runner, rt, world, local, K, Wm, step, ev_pairs=K)
    prog.check_errors()  # no tensor-core launch's bounded wait ran out
    dom_avg = sum(ev.ms(2 + 2 * k, 3 + 2 * k) for k in range(K)) / K
    ev.free()
    ms_step = _max_over_ranks(total_ms / K, world)
    peak, peak_kind = _peaks()
    if tensor:
        bmnk = launches[dom].info["mnk"]
        step_units = 2 * bmnk[0] * bmnk[1] * bmnk[2] * bmnk[3]
        value = world * step_units / (ms_step / 1e3) / 1e12
        achieved = step_units / (dom_avg / 1e3) / 1e12
        peak, peak_kind = _tf32x3_peak()
        unit = "TFLOP/s"
    else:
        step_units = step_bytes
        value = world * step_bytes / (ms_step / 1e3) / 1e9
        achieved = launches[dom].bytes / (dom_avg / 1e3) / 1e9
        unit = "GB/s"
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    tkey = name if name != "c3" or (shape or C3_DEFAULT) == C3_DEFAULT else f"c3_{'x'.join(map(str, shape))}"
    if os.path.exists(tpath):
        try:
            t = json.load(open(tpath)).get(tkey)
            if t and t.get("code_hash") == _code_hash(launches[dom].code):
                traffic = t["dram_bytes_per_launch"]
        except Exception:
            traffic = None
    roof = {"bound": "tensor" if tensor else "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_kind,
            "kernel": (f"{flat[dcall][1].name} (launch {dom}, {step_units} useful flops)" if tensor else
                       f"{launches[dom].kind} (launch {dom}, {launches[dom].bytes} algorithmic bytes)"),
            "kernel_ms": round(dom_avg, 4)}
    if tensor:
        pk_mhz = _sm_mhz_of_peak()
        if clk and pk_mhz:
            a_ghz = achieved / (clk["sm_mhz"] / 1e3)
            p_ghz = peak / (pk_mhz / 1e3)
            roof["per_sm_ghz"] = {"achieved": round(a_ghz, 2), "peak": round(p_ghz, 2), "frac": round(a_ghz / p_ghz, 4),
                                  "note": f"TFLOP/s per GHz of median SM clock: this run {clk['sm_mhz']:.0f} MHz, "
                                          f"the bf16 peak's sampling {pk_mhz:.0f} MHz"}
        roof["launch_tflops"] = round(step_units / (ms_step / 1e3) / 1e12, 1)
    elif traffic:
        roof["note"] = ("frac above 1 from L2 carry-over: DRAM traffic per launch is "
                        f"{traffic / launches[dom].bytes:.3f} of the algorithmic bytes") if achieved > peak else None

    # end to end through the public API: pinned host inputs -> device -> every launch -> outputs to host
    in_ids = list(name_of)
    h_in = {nid: rt.PinnedHost(inputs[name_of[nid]].nbytes) for nid in in_ids}
    for nid in in_ids:
        h_in[nid].array(inputs[name_of[nid]].size)[:] = inputs[name_of[nid]]
    out_sizes = {o: pkg.ir.size(fused.graph.nodes[o].shape) for o in outs}
    h_out = {o: rt.PinnedHost(out_sizes[o] * 4) for o in outs}
    h2d = sum(h.nbytes for h in h_in.values())
    d2h = sum(out_sizes[o] * 4 for o in outs)
    ke = max(1, min(K, args.e2e_steps))
    prog.free()
    # the public streaming API: every step copies its inputs in and its outputs out, overlapped across
    # consecutive steps (two device slots, separate copy-in / compute / copy-out streams)
    sp = rt.StreamedProgram(runner, fused.graph, lowered, in_ids, outs, slots=2)
    host_in = {nid: (h_in[nid].ptr, h_in[nid].nbytes) for nid in in_ids}
    host_out = {o: (h_out[o].ptr, out_sizes[o] * 4) for o in outs}
    for _ in range(2):
        sp.submit(host_in, host_out)
    sp.drain()
    _barrier(world)
    sp.mark("start")
    for _ in range(ke):
        sp.submit(host_in, host_out)
    sp.mark("end")
    sp.drain()
    e2e_ms = _max_over_ranks(sp.elapsed_ms() / ke, world)
    sp.free()
    scale = 1e12 if tensor else 1e9
    e2e_value = world * step_units / scale / (e2e_ms / 1e3)
    ceil = copy_ceiling(rt, runner, list(h_in.values()), list(h_out.values()))
    ceil["value"] = round(world * step_units / scale / (ceil["both_ms"] / 1e3), 2)
    ceil["frac"] = round(e2e_value / ceil["value"], 4)
    for h in list(h_in.values()) + list(h_out.values()):
        h.free()
    rec = {
        "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": K, "warmup": Wm,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (mulberry32 seed 0, Box-Muller normals)",
        "config": {**cfg, "parallelism": f"replicas x{world}" if world > 1 else "1 GPU",
                   "bytes_per_step": step_bytes, "launches_per_step": len(launches),
                   "units": "the reference fused plan's algorithmic bytes per step (amendment 33), as the "
                            "reference arm counts them" if not tensor else "useful matmul flops per step",
                   "bytes_moved_per_step": moved_bytes,
                   "moved_gbs": round(world * moved_bytes / (ms_step / 1e3) / 1e9, 1)},
        "roofline": roof,
        "e2e": {"value": round(e2e_value, 2), "unit": unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 3), "steps": ke, "ceiling": ceil,
                "api": "StreamedProgram: per step H2D of every input from pinned memory, the launches, D2H of every "
                       "output; consecutive steps overlap their copies"},
        "gpu_launches": K * prog.kernel_launches,
        "clocks": clk,
    }
    if cpu and rank == 0 and world == 1 and not args.no_cpu:
        rec["cpu_baseline"] = cpu_baseline(name, pkg, cg, wl, args.cpu_seconds, variant, shape)
    return rec


def _tf32x3_peak():
    """3xTF32 useful-flop ceiling: TF32 dense = half the measured bf16 dense rate (the nominal 1.1 : 2.25 PF), / 3."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            bf16 = float(json.load(f)["bf16_tflops"])
        return round(bf16 / 2 / 3, 1), "measured bf16 burst / 2 (tf32) / 3 (3xTF32)"
    except Exception:
        return round(1590.0 / 2 / 3, 1), "fallback bf16 1.59 PF / 2 / 3"


def step_roofline(launches, hbm_gbs, tensor_tflops):
    """The ideal time of a whole step: every launch at its own roofline -- a GEMM at the slower of its
    useful flops / the tensor ceiling and its algorithmic bytes / HBM, every other launch at its
    algorithmic bytes / HBM -- summed in milliseconds, with the split into the two kinds."""
    t_tensor = t_hbm = 0.0
    flops = nbytes = 0
    for lau in launches:
        info = getattr(lau, "info", None) or {}
        if "mnk" in info:
            b, M, K, N = info["mnk"]
            f = 2 * b * M * N * K
            flops += f
            t_tensor += max(f / (tensor_tflops * 1e12), lau.bytes / (hbm_gbs * 1e9))
        else:
            t_hbm += lau.bytes / (hbm_gbs * 1e9)
        nbytes += lau.bytes
    return {"ideal_ms": round((t_tensor + t_hbm) * 1e3, 3), "gemm_ms": round(t_tensor * 1e3, 3),
            "hbm_ms": round(t_hbm * 1e3, 3), "matmul_tflop": round(flops / 1e12, 3), "algorithmic_gb": round(nbytes / 1e9, 2)}


def _sustained_peaks():
    """(HBM GB/s, 3xTF32 TFLOP/s) for a kernel timed inside a long step: the measured copy rate and the
    measured sustained bf16 dense rate / 2 / 3."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])) / 6, "measured"
    except Exception:
        return 6650.0, 1400.0 / 6, "fallback"


def _code_hash(code):
    """Hash of a launch's source plus the code of every library template it includes (their `//`
    comments and blank lines left out), so a recorded traffic figure is used only for the exact
    kernel it was captured on, and a comment edit does not orphan it."""
    import hashlib
    import re
    h = hashlib.sha256(code.encode())
    tdir = os.path.join(ROOT, "tensor-compiler-webgpu_b200", "csrc", "templates")
    for name in sorted(set(re.findall(r'#include "tcb/([a-z_]+\.cuh)"', code))):
        with open(os.path.join(tdir, name)) as f:
            text = f.read()
        lines = (ln.rstrip() for ln in re.sub(r"//[^\n]*", "", text).splitlines())
        h.update("\n".join(ln for ln in lines if ln).encode())
    return h.hexdigest()[:16]


def cpu_baseline(name, pkg, cg, wl, seconds, variant=None, shape=None):
    """The oracle (C restatement of interp.js, 1 core, -O2) on a bounded row sample; same unit rule."""
    oracle = _oracle()
    M = (shape or C3_DEFAULT)[0]
    full = {"c2": 8192, "c4": 65536, "c3": M}[name]
    rows = 8 if name != "c3" else 1
    while True:
        graph, inputs, units = cpu_sample(name, wl, pkg, cg, rows, variant, shape)
        t0 = time.perf_counter()
        oracle.evaluate(graph, inputs, want=[])
        dt = time.perf_counter() - t0
        if dt * 2 > seconds or rows >= full:
            break
        rows = min(full, max(rows * 2, int(rows * seconds / max(dt, 1e-3) / 1.5)))
    if name == "c3":
        return {"value": round(units / dt / 1e12, 6), "unit": "TFLOP/s", "cores": 1, "kind": "port",
                "sample": f"{rows} of {M} rows of A (the interpreter is linear in M), triple loop once in {dt:.2f} s "
                          f"(C restatement of interp.js, float64, single thread, gcc -O2)", "seconds": round(dt, 3)}
    return {"value": round(units / dt / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{rows} of {full} rows, whole graph evaluated once in {dt:.2f} s "
                      f"(C restatement of interp.js, float64, single thread, gcc -O2)",
            "seconds": round(dt, 3)}


def run_reference(args):
    """The reference's CPU implementation of the path (the oracle port), all host threads, rank 0 only.

    The headline is C2 (the same workload, metric and unit as this repository's line); with the default
    workload the other configs follow as records, one bounded sample each."""
    world, rank, local = _dist()
    if rank != 0:
        return
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    head = "c2" if args.workload == "all" else args.workload
    with ctx.Pool(cores) as pool:
        out = _reference_line(args, pool, cores, head, steps=args.steps, warmup=args.warmup)
        if args.workload == "all":
            out["records"] = {
                "c1": _reference_line(args, pool, cores, "c1", steps=3, warmup=1),
                "c3": _reference_line(args, pool, cores, "c3", steps=1, warmup=1),
                "c4": _reference_line(args, pool, cores, "c4", steps=2, warmup=1),
                "train": _reference_line(args, pool, cores, "c5", steps=1, warmup=1)}
    print(json.dumps(out), flush=True)


def _reference_line(args, pool, cores, name, steps, warmup):
    rows = {"c2": 64, "c4": 16, "c3": 1, "c1": 1, "c5": 1}[name]
    job = (name, rows, 1, None, None)
    # every worker prepares its sample once (untimed); a step is every worker evaluating it once
    pool.map(_cpu_worker, [job] * cores, chunksize=1)
    times, total = [], 0
    for k in range(warmup + steps):
        res = pool.map(_cpu_worker, [job] * cores, chunksize=1)
        if k >= warmup:
            times.append(max(t for _, t in res))
            total += sum(b for b, _ in res)
    wall = sum(times)
    unit, scale = {"c1": ("samples/s", 1), "c5": ("tokens/s", 1), "c3": ("TFLOP/s", 1e-12)}.get(name, ("GB/s", 1e-9))
    value = total / wall * scale
    what = {"c1": "the whole C1 step graph", "c5": "1 sequence of the C5 training step (forward, backward, Adam)"}
    full = {"c2": 8192, "c4": 65536, "c3": 4096}.get(name)
    sample = (f"{cores} processes x " + (what[name] if name in what else f"{rows} of {full} rows") +
              " per step, step time = slowest process (C restatement of interp.js, float64)")
    return {"impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": unit, "n_gpus": 1,
            "steps": steps, "warmup": warmup, "ms_per_step": round(1e3 * wall / len(times), 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (mulberry32 seed 0)",
            "config": {"workload": {"c2": "C2 elementwise chain fp32 [8192,8192] fwd+bwd",
                                    "c4": "C4 softmax fp32 [65536,4096] fwd+bwd, 1% rows +800",
                                    "c3": "C3 matmul [4096,4096]x[4096,4096] + bias + relu (fp32 via 3xTF32)",
                                    "c1": "C1 MLP 64->32->10 tanh, batch 64, fwd+bwd",
                                    "c5": "C5 decoder transformer train step (fwd+bwd+Adam)"}[name]},
            "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_sweep(args):
    """The amendment-34 sweep and the copy/read ceilings under amendment 32's protocol (not the driver's line)."""
    tm = importlib.import_module(PKG + ".timing")
    rt = importlib.import_module(PKG + ".runtime")
    codes = set()
    for w in tm.workloads():
        if args.only and not any(x in w["id"] for x in args.only.split(",")):
            continue
        for prog in tm.build_variants(w)["programs"].values():
            codes |= {d["code"] for d in prog["dispatches"]}
    codes |= {c["program"]["dispatches"][0]["code"] for c in tm.ceiling_programs()}
    rt.precompile(codes)
    bench = tm.Bench.create(0)
    out = open(args.sweep, "w")

    def log(rec):
        out.write(json.dumps(rec) + "\n")
        out.flush()
        if rec["family"] == "ceiling":
            print(f"{rec['id']:32s} {rec['GBps']:9.1f} GB/s", flush=True)
        elif rec.get("failedGate"):
            print(f"{rec['id']:36s} GATE FAILED for {rec['failedGate']}: not timed", flush=True)
        else:
            v = "  ".join(f"{k} {d['GBps']:8.1f} GB/s ({d['launches']})" for k, d in rec["variants"].items())
            print(f"{rec['id']:36s} {v}", flush=True)
    oracle = _oracle()  # the checker of the sweep's gate, never the thing timed

    def judge(graph, inputs, outputs, gpu):
        values, bounds, _ = oracle.reference_with_bounds(graph, inputs, want=list(outputs))
        return oracle.judge_outputs([values[o] for o in outputs], [bounds[o] for o in outputs], gpu)
    res = tm.run_sweep(bench, only=args.only.split(",") if args.only else None, log=log, judge=judge)
    out.close()
    bench.close()
    leaks = [r["id"] for r in res if r["created"]]
    ungated = [r["id"] for r in res if r["family"] != "ceiling" and not r["gate"]["pass"]]
    print(json.dumps({"sweep": len(res), "objects_created_in_timed_regions": leaks, "failed_gate": ungated}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="all", choices=["all", "c1", "c2", "c4", "c3", "c5"])
    ap.add_argument("--batch", type=int, default=None, help="C5 global batch (default 512)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10,
                    help="steps of the end-to-end measurement (copies overlap across steps: the first step's "
                         "input copy and the last one's output copy are the pipeline's fill and drain)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--rows", type=int, default=None, help="cut C2/C4 to fewer rows (profiling cases only)")
    ap.add_argument("--sweep", default=None, help="run the amendment-34 sweep, one JSON record per line to this file")
    ap.add_argument("--only", default=None, help="sweep: comma-separated id substrings")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.sweep:
        run_sweep(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    world, rank, local = _dist()
    _init_group(world)
    pkg, rt, cg, wl = _mods()
    runner = rt.GpuRunner.create(local)
    try:
        if args.workload == "all":
            out = graph_record(args, "c2", runner, world, rank, local)
            recs = {}
            if world == 1:
                sub = argparse.Namespace(**{**vars(args), "cpu_seconds": min(args.cpu_seconds, 5.0)})
                recs["c1"] = c1_record(sub, runner, rank)
                for shape in wl.C3_SHAPES:
                    for act in ("relu", "tanh"):
                        recs[f"c3_{'x'.join(map(str, shape))}_{act}"] = graph_record(
                            sub, "c3", runner, world, rank, local, variant=act, shape=shape,
                            cpu=(act == "relu"))
                for what in ("softmax", "logsoftmax"):
                    recs[f"c4_{what}"] = graph_record(sub, "c4", runner, world, rank, local, variant=what,
                                                      cpu=(what == "softmax"))
            recs["train"] = c5_record(argparse.Namespace(**{**vars(args), "cpu_seconds": min(args.cpu_seconds, 5.0)}),
                                      runner, world, rank, local)
            out["records"] = recs
            out["gpu_launches"] = out["gpu_launches"] + sum(r.get("gpu_launches", 0) for r in recs.values())
        elif args.workload == "c5":
            out = c5_record(args, runner, world, rank, local)
        elif args.workload == "c1":
            out = c1_record(args, runner, rank)
        else:
            out = graph_record(args, args.workload, runner, world, rank, local)
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        runner.close()
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


def _collective(tr, world):
    if world == 1:
        return "none (1 rank)"
    if tr.buckets == 1:
        return f"one NCCL sum-allreduce of the flat gradient buffer ({tr.flat_floats * 4} bytes) after the backward"
    return (f"{len(tr.bucket_spans)} NCCL sum-allreduces of the flat gradient buffer's buckets "
            f"({[hi - lo for lo, hi in tr.bucket_spans]} bytes), each issued on a collective stream as soon as "
            f"the backward has written it, overlapping the rest of the backward")


def c5_record(args, runner, world, rank, local):
    """C5: the decoder transformer's training step, data parallel over the batch (tokens/s): every rank
    runs the gradient program on its shard, the library's NCCL communicator sums the gradients (the
    flat gradient buffer in buckets, each reduced as soon as the backward has written it), every rank
    runs the same Adam program."""
    pkg, rt, cg, wl = _mods()
    dp = importlib.import_module(PKG + ".dp")
    cfg, c = wl.c5_cfg(batch=args.batch or wl.C5_CONFIG["batch"])
    V, B, T = c["V"], c["batch"], cfg["T"]
    if B % world:
        raise SystemExit(f"global batch {B} does not split over {world} ranks")
    bl = B // world
    comm = dp.Comm(runner, rank, world) if world > 1 else None
    params = pkg.steps.init_params_normal(V, 0, 0.02, cfg)
    tr = dp.DPTrainer(runner, V, bl, cfg, params, comm=comm, capture=True)
    toks = wl.c5_tokens(B, T, V, seed=0)[rank * bl:(rank + 1) * bl]
    x, y = wl.one_hot_batch(toks, V)
    tr.grad_prog.write(tr.x_id, x)
    tr.grad_prog.write(tr.y_id, y)
    K, Wm = args.steps, args.warmup

    def step(k, ev):
        tr.step_device()
    # the allreduce runs on the library's stream inside each step; a step's end is the end of its Adam program
    total_ms, ev, clk = _timed(runner, rt, world, local, K, Wm, step)
    ev.free()
    if comm:
        comm.wait()
    tr.grad_prog.check_errors()
    tr.adam_prog.check_errors()
    ms = _max_over_ranks(total_ms / K, world)
    tokens = B * T
    value = tokens / (ms / 1e3)
    flops = _matmul_flops(pkg, tr.fg.graph) * world
    hbm, tfl, peak_kind = _sustained_peaks()
    sr = step_roofline(list(tr.grad_prog.launches) + list(tr.adam_prog.launches), hbm, tfl)
    # end to end: this rank's x, y from pinned host memory, the step, the loss back to the host
    hx, hy = rt.PinnedHost(x.nbytes), rt.PinnedHost(y.nbytes)
    hx.array(x.size)[:] = x
    hy.array(y.size)[:] = y
    hl = rt.PinnedHost(4)
    lib = rt.lib()

    def e2e(k, ev):
        tr.grad_prog.write_async(tr.x_id, hx.ptr, x.nbytes)
        tr.grad_prog.write_async(tr.y_id, hy.ptr, y.nbytes)
        tr.step_device()
        rt.check(lib.tc_memcpy_dtoh(runner.ctx, hl.ptr, tr.grad_prog.ptr(tr.loss_id), 4))
    ke = max(1, min(K, args.e2e_steps))
    e2e_total, ev2, _ = _timed(runner, rt, world, local, ke, 1, e2e)
    ev2.free()
    if comm:
        comm.wait()
    e2e_ms = _max_over_ranks(e2e_total / ke, world)
    coll_ms = None
    if comm:
        # the whole flat gradient buffer reduced alone, every rank the same calls: what the collective
        # would cost the step if nothing overlapped it
        def ar(k, ev):
            comm.allreduce_mean(tr.flat.ptr, tr.flat_floats, prescaled=tr.prescaled)
        ar_total, ev3, _ = _timed(runner, rt, world, local, 10, 3, ar)
        ev3.free()
        comm.wait()
        coll_ms = _max_over_ranks(ar_total / 10, world)
    rec = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": Wm,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic tokens uniform 0..64 (mulberry32 seed 0), weights N(0,0.02)",
        "config": {"workload": "C5 decoder transformer train step (fwd+bwd+Adam)", "V": V, "d": cfg["d"],
                   "L": cfg["L"], "H": cfg["H"], "ff": cfg["ff"], "seq_len": T, "global_batch": B,
                   "parallelism": f"dp{world}", "collective": _collective(tr, world),
                   "launches_per_step": tr.kernel_launches,
                   "arena_bytes": tr.grad_prog.arena_bytes + tr.adam_prog.arena_bytes,
                   "l2": "activations > L2 (each [B*T, ff] tensor 512 MiB at one rank)"},
        "roofline": {"bound": "tensor", "achieved": round(flops / (ms / 1e3) / 1e12, 2), "peak": round(tfl * world, 1),
                     "unit": "TFLOP/s", "frac": round(flops / (ms / 1e3) / 1e12 / (tfl * world), 4), "traffic": None,
                     "kernel": "whole step: matmul FLOPs / step time against the sustained 3xTF32 ceiling x ranks"},
        "step_roofline": dict(sr, frac=round(sr["ideal_ms"] / ms, 4), peaks=f"{peak_kind}: HBM {hbm:.1f} GB/s, "
                              f"3xTF32 {tfl:.1f} TFLOP/s (sustained bf16 / 2 / 3)",
                              how="per rank: each launch of the gradient and Adam programs at its own roofline, summed"),
        "e2e": {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": 2 * x.nbytes,
                "d2h_bytes_per_step": 4, "ms_per_step": round(e2e_ms, 3)},
        "gpu_launches": K * tr.kernel_launches,
        "clocks": clk,
    }
    gap = ms - sr["ideal_ms"]
    if coll_ms is not None:
        rec["collective"] = {"allreduce_alone_ms": round(coll_ms, 3), "bytes": tr.flat_floats * 4,
                             "buckets": len(tr.bucket_spans) if tr.buckets > 1 else 1}
    rec["limiter"] = (f"per-rank kernels: the step takes {ms:.3f} ms against {sr['ideal_ms']:.3f} ms with every "
                      f"launch at its own roofline ({gap:.3f} ms above it, {tr.kernel_launches} launches)"
                      + (f"; the gradient allreduce alone takes {coll_ms:.3f} ms, "
                         + (f"{len(tr.bucket_spans) - 1} of its {len(tr.bucket_spans)} buckets overlapping the "
                            f"backward" if tr.buckets > 1 else "after the backward") if coll_ms is not None else ""))
    if rank == 0 and world == 1 and not args.no_cpu:
        oracle = _oracle()
        graph, inputs, units = cpu_sample("c5", wl, pkg, cg, 1)
        t0 = time.perf_counter()
        oracle.evaluate(graph, inputs, want=[])
        dt = time.perf_counter() - t0
        rec["cpu_baseline"] = {"value": round(units / dt, 1), "unit": "tokens/s", "cores": 1, "kind": "port",
                               "sample": f"1 sequence (256 tokens) of the full training step (forward, backward, "
                                         f"Adam) in {dt:.2f} s (C restatement of interp.js, float64, single thread)"}
    for h in (hx, hy, hl):
        h.free()
    tr.destroy()
    if comm:
        comm.destroy()
    return rec


def c1_record(args, runner, rank):
    """C1: the MLP 64 -> 32 -> 10 (tanh) step, batch 64, forward + backward fused; samples/s (launch-bound)."""
    pkg, rt, cg, wl = _mods()
    step = wl.c1_step(64)
    inputs = wl.c1_inputs(64)
    inputs[step["cotangent"]] = [1.0]
    keep = [step["loss"], *step["outputs"].values()]
    fused = pkg.fuse.fuse(step["graph"], keep=keep)
    outs = [fused.index[k] for k in dict.fromkeys(keep)]
    # the trainers' resident lowering: sums and elementwise readers in their producers' passes
    lowered = cg.lower_fused(fused.graph, matmul="naive", colfuse=True, mofuse=True, keep=outs)
    prog = rt.Program(runner, fused.graph, lowered, keep=outs)
    name_of = {n.id: n.attrs["name"] for n in fused.graph.nodes if n.op == "input"}
    for nid, nm in name_of.items():
        prog.write(nid, inputs[nm])
    prog.capture()
    K, Wm = max(args.steps, 100), args.warmup
    total_ms, ev, clk = _timed(runner, rt, 1, 0, K, Wm, lambda k, ev: prog.run())
    ev.free()
    us = total_ms / K * 1e3
    # end to end: x, y from pinned host memory, the step, the loss and the gradients back
    xin = [nid for nid, nm in name_of.items() if nm in ("x", "y")]
    hosts = {nid: rt.PinnedHost(np.asarray(inputs[name_of[nid]], np.float32).nbytes) for nid in xin}
    for nid in xin:
        hosts[nid].array(hosts[nid].nbytes // 4)[:] = np.asarray(inputs[name_of[nid]], np.float32).reshape(-1)
    osz = {o: pkg.ir.size(fused.graph.nodes[o].shape) for o in outs}
    hout = {o: rt.PinnedHost(osz[o] * 4) for o in outs}
    lib = rt.lib()

    def e2e(k, ev):
        for nid in xin:
            prog.write_async(nid, hosts[nid].ptr, hosts[nid].nbytes)
        prog.run()
        for o in outs:
            rt.check(lib.tc_memcpy_dtoh(runner.ctx, hout[o].ptr, prog.ptr(o), osz[o] * 4))
    e2e_total, ev2, _ = _timed(runner, rt, 1, 0, K, 3, e2e)
    ev2.free()
    e2e_us = e2e_total / K * 1e3
    rec = {"metric": METRIC, "value": round(64 / (us / 1e6), 1), "unit": "samples/s", "n_gpus": 1,
           "steps": K, "warmup": Wm, "ms_per_step": round(us / 1e3, 5), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic (features int(0..16)/16, labels 0..9, Glorot weights)",
           "config": {"workload": "C1 MLP 64->32->10 tanh, batch 64, fwd+bwd (fused, one CUDA graph)",
                      "launches_per_step": prog.kernel_launches, "us_per_step": round(us, 2)},
           "roofline": {"bound": "launch", "achieved": round(us / prog.kernel_launches, 3), "peak": None,
                        "unit": "us per kernel", "frac": None, "traffic": None,
                        "kernel": "whole step (launch-latency bound: tens of tiny kernels)"},
           "e2e": {"value": round(64 / (e2e_us / 1e6), 1), "unit": "samples/s",
                   "h2d_bytes_per_step": sum(h.nbytes for h in hosts.values()),
                   "d2h_bytes_per_step": sum(osz[o] * 4 for o in outs), "us_per_step": round(e2e_us, 2)},
           "gpu_launches": K * prog.kernel_launches, "clocks": clk}
    if rank == 0 and not args.no_cpu:
        oracle = _oracle()
        graph = step["graph"]
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 5.0):
            oracle.evaluate(graph, inputs, want=[])
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        rec["cpu_baseline"] = {"value": round(64 / dt, 1), "unit": "samples/s", "cores": 1, "kind": "port",
                               "sample": f"the whole step graph, {reps} evaluations (C restatement of interp.js)"}
    for h in list(hosts.values()) + list(hout.values()):
        h.free()
    prog.free()
    return rec


def _matmul_flops(pkg, graph):
    flops = 0
    for n in graph.nodes:
        if n.op == "fused" and n.attrs["kind"] == "epilogue":
            b = pkg.fuse.body_of(n)
            r = next(x for x in b.nodes if x.op == "matmul")
            a_s, b_s = b.nodes[r.inputs[0]].shape, b.nodes[r.inputs[1]].shape
        elif n.op == "matmul":
            a_s, b_s = graph.nodes[n.inputs[0]].shape, graph.nodes[n.inputs[1]].shape
        else:
            continue
        flops += 2 * pkg.ir.size(a_s[:-2]) * a_s[-2] * a_s[-1] * b_s[-1]
    return flops


if __name__ == "__main__":
    main()
