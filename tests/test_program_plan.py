"""Resident programs built on the CPU against a recording stand-in of the device library.

`Program` turns a lowered graph into a native plan: arena offsets from value lifetimes, reshapes
aliased, small same-source launches hoisted and batched (`batch=True`), the weights' operand splits
hoisted into one launch, per-launch control blocks.  These tests build the trainers' real programs
with `lib()` replaced by a recorder (device addresses from a bump allocator; the arena planner is
the library's own `tc_plan_memory`, which needs no device) and then replay the recorded order on
the host, tracking which value each byte of device memory holds:

* every launch reads only values that are still in place (no arena reuse clobbers a live value, in
  the reordered, batched plan as in the plain one);
* the launches batched together neither read nor overlap one another's outputs;
* the argument tables uploaded for batched launches and hoisted splits carry the right addresses.
"""
import ctypes
import importlib

import numpy as np
import pytest


class Recorder:
    """The subset of the C ABI a Program uses, recorded instead of executed."""

    def __init__(self, real):
        self.real = real
        self.next_addr = 1 << 40
        self.buffers = {}          # handle -> (address, bytes)
        self.uploads = {}          # address -> bytes uploaded
        self.plans = {}            # plan handle -> entries
        self._h = 100

    def _handle(self):
        self._h += 1
        return self._h

    def tc_last_error(self):
        return b"recorder"

    def tc_alloc(self, ctx, nbytes, canary, out):
        h = self._handle()
        addr = self.next_addr
        self.next_addr += (int(nbytes) + 255) // 256 * 256 + 256
        self.buffers[h] = (addr, int(nbytes))
        out._obj.value = h
        return 0

    def tc_buf_ptr(self, h, out):
        out._obj.value = self.buffers[h if isinstance(h, int) else h.value][0]
        return 0

    def tc_free(self, h):
        return 0

    def tc_memset32(self, ctx, ptr, value, count):
        return 0

    def tc_upload(self, h, host, nbytes, offset):
        addr = self.buffers[h if isinstance(h, int) else h.value][0]
        self.uploads[addr + int(offset)] = ctypes.string_at(host, int(nbytes))
        return 0

    def tc_memcpy_htod(self, ctx, dst, host, nbytes):
        return 0

    def tc_sync(self, ctx, timeout):
        return 0

    def tc_plan_create(self, ctx, out):
        h = self._handle()
        self.plans[h] = []
        out._obj.value = h
        return 0

    def _args(self, a):
        a = a._obj
        return {"in": list(a.in_), "out": a.out, "scratch": a.scratch, "p": list(a.p)}

    def tc_plan_add_launch(self, plan, mod, name, grid, block, smem, args):
        self.plans[plan.value].append(("launch", name.decode(), tuple(grid), self._args(args), None))
        return 0

    def tc_plan_add_launch_tma(self, plan, mod, name, grid, block, smem, n, desc, args):
        maps = [tuple(desc[8 * m + j] for j in range(8)) for m in range(n)]
        self.plans[plan.value].append(("launch", name.decode(), tuple(grid), self._args(args), maps))
        return 0

    def tc_plan_add_copy(self, plan, dst, src, nbytes):
        self.plans[plan.value].append(("copy", int(dst), int(src), int(nbytes)))
        return 0

    def tc_plan_add_allreduce(self, plan, comm, buf, count, scale):
        self.plans[plan.value].append(("allreduce", int(buf), int(count), float(scale.value), comm))
        return 0

    def tc_plan_capture(self, plan):
        return 0

    def tc_plan_free(self, plan):
        return 0

    def tc_plan_memory(self, *a):
        return self.real.tc_plan_memory(*a)


@pytest.fixture()
def recorded(pkg, monkeypatch):
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    rec = Recorder(rt.lib())
    monkeypatch.setattr(rt, "lib", lambda: rec)
    monkeypatch.setattr(rt.GpuRunner, "pipeline", lambda self, code: rt.Module(hash(code) & 0xFFFF, self))
    return rt, rec, rt.GpuRunner(1, 0)


def _replay(prog, graph):
    """Walk the program's launches in plan order, tracking which value each byte range holds."""
    nodes = graph.nodes

    def root(i):
        while i in prog.alias:
            i = prog.alias[i]
        return i

    def rng(i):
        r = root(i)
        return prog.ptrs[r], prog.ptrs[r] + max(1, int(np.prod(nodes[r].shape, dtype=np.int64))) * 4

    holder = []        # (lo, hi, node) of values in memory
    valid = set()
    for n in nodes:
        if n.op in ("input", "const") and n.id in prog.ptrs:
            holder.append((*rng(n.id), root(n.id)))
            valid.add(root(n.id))

    def write(i):
        lo, hi = rng(i)
        for (a, b, v) in list(holder):
            if a < hi and lo < b and v != root(i):
                valid.discard(v)
        holder.append((lo, hi, root(i)))
        valid.add(root(i))

    for lau in prog.launches:
        members = getattr(lau, "members", [lau])
        outs = [n for m in members for n in (getattr(m, "nodes", None) or [m.node])]  # two-output launches too
        for m in members:
            for i in m.inputs:
                if nodes[root(i)].op in ("input", "const"):
                    continue
                assert root(i) in valid, f"launch of node {m.node} reads node {i} after its memory was reused"
        if len(members) > 1:
            spans = [rng(o) for o in outs]
            reads = [rng(i) for m in members for i in m.inputs]
            for k, (a, b) in enumerate(spans):
                for j, (c, d) in enumerate(spans):
                    assert j == k or b <= c or d <= a, "batched outputs overlap"
                for (c, d) in reads:
                    if c < b and a < d:
                        assert (c, d) == (a, b), "a batched launch writes what another member reads"
        for o in outs:
            write(o)


def _dp_trainer(pkg, runner, batch, full=False, comm=None, buckets=None):
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    dp = importlib.import_module("tensor-compiler-webgpu_b200.dp")
    cfg, c = wl.c5_cfg(batch=512) if full else wl.c5_cfg(d=64, L=2, H=4, ff=128, T=32, batch=4)
    V, B = c["V"], c["batch"]
    params = pkg.steps.init_params_normal(V, 0, 0.02, cfg)
    return dp.DPTrainer(runner, V, B, cfg, params, batch=batch, capture=False, comm=comm, buckets=buckets)


class _FakeComm:
    def __init__(self, world):
        self.world, self.handle = world, ctypes.c_void_p(0x5eed)


@pytest.mark.parametrize("batch,full", [(False, False), (True, False), (True, True)])
def test_plans_never_read_a_reused_value(pkg, recorded, batch, full):
    """Small model plain and batched, and the C5 benchmark's own programs (global batch 512)."""
    rt, rec, runner = recorded
    tr = _dp_trainer(pkg, runner, batch, full)
    _replay(tr.grad_prog, tr.fg.graph)
    _replay(tr.adam_prog, tr.fa.graph)


def test_batched_plan_tables_and_hoisted_splits(pkg, recorded):
    rt, rec, runner = recorded
    tr = _dp_trainer(pkg, runner, True)
    ap = tr.adam_prog
    multis = [l for l in ap.launches if isinstance(l, rt.MultiLaunch)]
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    assert multis and 2 * len(ap.launches) < len(cg.lower_fused(tr.fa.graph, matmul="tiled")["launches"])
    entries = rec.plans[ap.plan.value]
    launches = [e for e in entries if e[0] == "launch"]
    assert len(launches) == ap.kernel_launches
    # each batched launch's table: one argument block per member, with that member's addresses
    multi_calls = [e for e in launches if e[1] == "tcb_elementwise_multi"]
    for lau in multis:
        call = next(e for e in multi_calls if e[2][1] == len(lau.members)
                    and rec.uploads.get(e[3]["scratch"]) is not None
                    and rt.Args.from_buffer_copy(rec.uploads[e[3]["scratch"]][:ctypes.sizeof(rt.Args)]).out
                    == ap.ptrs[lau.members[0].node])
        raw = rec.uploads[call[3]["scratch"]]
        table = (rt.Args * len(lau.members)).from_buffer_copy(raw)
        for j, m in enumerate(lau.members):
            assert table[j].out == ap.ptrs[m.node]
            assert [table[j].in_[k] for k in range(len(m.inputs))] == [ap.ptrs[i] for i in m.inputs]
            assert table[j].p[0] == m.calls[0].params[0]
    # the gradient program: one up-front split launch whose jobs read the weights and fill the
    # buffers the hoisted GEMMs' B maps point at; those GEMMs issue no split_b of their own
    gp = tr.grad_prog
    assert gp.hoisted
    g_entries = [e for e in rec.plans[gp.plan.value] if e[0] == "launch"]
    assert g_entries[0][1] == "tcb_split_multi"
    jobs = np.frombuffer(rec.uploads[g_entries[0][3]["scratch"]], dtype=np.uint64).reshape(-1, 8)
    assert len(jobs) == len(gp.hoisted)
    split_targets = {(int(j[1]), int(j[2])) for j in jobs}
    assert split_targets == set(gp.hoisted.values())
    for k, (hi, lo) in gp.hoisted.items():
        lau = gp.launches[k]
        b = lau.inputs[lau.info["ib"]]
        assert any(int(j[0]) == gp.ptrs[b] and (int(j[1]), int(j[2])) == (hi, lo) for j in jobs)
    gemms = [e for e in g_entries if e[1] == "tcb_gemm_tc"]
    hoisted_maps = [e[4] for e in gemms if (e[4][2][0], e[4][3][0]) in split_targets]
    assert len(hoisted_maps) == len(gp.hoisted)
    n_split_b = sum(1 for e in g_entries if e[1] == "tcb_split_b")
    n_split_b_lowered = sum(1 for lau in gp.launches for c in lau.calls if c.name == "tcb_split_b")
    assert n_split_b == n_split_b_lowered - len(gp.hoisted)
    # no one-block clearing launches in a resident plan; every GEMM has its own control block
    assert all(e[1] != "tcb_gemm_prep" for e in g_entries)
    ctrl = [e[3]["p"][15] for e in gemms]
    assert len(set(ctrl)) == len(ctrl) and all(c for c in ctrl)


def test_replay_catches_a_clobbered_value(pkg, recorded, monkeypatch):
    """The replay is not vacuous: with an arena planner that puts every value at offset 0 it finds a
    hazard (batched outputs on top of one another, or a launch reading a value whose memory was
    reused)."""
    rt, rec, runner = recorded

    def all_at_zero(n, nbytes, first, last, offsets, total):
        for k in range(n):
            offsets[k] = 0
        total._obj.value = max(int(nbytes[k]) for k in range(n)) if n else 0
        return 0

    monkeypatch.setattr(rec, "tc_plan_memory", all_at_zero)
    tr = _dp_trainer(pkg, runner, True)
    with pytest.raises(AssertionError, match="memory was reused|overlap"):
        _replay(tr.grad_prog, tr.fg.graph)


@pytest.mark.parametrize("world,buckets,full", [(4, 4, False), (8, 4, True), (3, 2, False), (2, 1, False)])
def test_bucketed_allreduce_plan(pkg, recorded, world, buckets, full):
    """Data parallel with the gradient buckets reduced during the backward: the buckets tile the flat
    gradient buffer exactly, each allreduce is planned after every launch that writes a gradient of its
    bucket, and no launch after it reads or writes its range (it runs on another stream meanwhile).
    Power-of-two worlds reduce a plain sum (the 1/W is in the cotangent seed), others scale by 1/W."""
    rt, rec, runner = recorded
    tr = _dp_trainer(pkg, runner, True, full, comm=_FakeComm(world), buckets=buckets)
    gp = tr.grad_prog
    entries = rec.plans[gp.plan.value]
    colls = [(k, e) for k, e in enumerate(entries) if e[0] == "allreduce"]
    if buckets == 1:
        assert not colls and tr.buckets == 1
        return
    assert 2 <= len(colls) <= buckets
    base = tr.flat.ptr
    spans = sorted((e[1] - base, e[1] - base + 4 * e[2]) for _, e in colls)
    assert spans[0][0] == 0 and spans[-1][1] == 4 * tr.flat_floats
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    want_scale = float(np.float32(1.0 if world & (world - 1) == 0 else 1.0 / world))
    assert all(e[3] == want_scale for _, e in colls)
    grads = [tr.fg.index[tr.gs["grads"][n]] for n in tr.names]
    nbytes = {g: 4 * int(np.prod(tr.fg.graph.nodes[g].shape, dtype=np.int64)) for g in grads}
    launch_entries = [k for k, e in enumerate(entries) if e[0] == "launch"]
    assert len(launch_entries) == gp.kernel_launches

    def touches(e, lo, hi):
        a = e[3]
        ptrs = [a["out"], *[p for p in a["in"] if p]]
        if e[1] == "tcb_elementwise_mo":
            ptrs += [p for p in a["p"][1:4] if p]
        return any(lo <= p < hi for p in ptrs)
    for k, e in colls:
        lo, hi = e[1], e[1] + 4 * e[2]
        members = [g for g in grads if lo <= gp.ptrs[g] < hi]
        assert members and all(gp.ptrs[g] + nbytes[g] <= hi for g in members)
        assert any(touches(entries[j], lo, hi) for j in launch_entries if j < k)
        for j in launch_entries:
            if j > k:
                assert not touches(entries[j], lo, hi), (k, j, entries[j][1])
    # the layout follows the order in which the backward finishes the gradients
    at = [gp.ptrs[tr.fg.index[tr.gs["grads"][n]]] for n in tr.order]
    assert at == sorted(at)


@pytest.mark.parametrize("sizes,buckets", [([100, 300, 1000, 4, 5000, 256], 4), ([100], 4), ([100, 200], 1),
                                           ([4096] * 58, 4), ([262144 * 4, 1024, 1024, 262144 * 4], 3)])
def test_bucket_layout(sizes, buckets):
    """The flat gradient buffer's layout: 256-byte aligned slices back to back, at most `buckets`
    contiguous spans that cover it exactly, each cut at a tensor boundary."""
    dp = importlib.import_module("tensor-compiler-webgpu_b200.dp")
    offs, spans = dp.bucket_layout(sizes, buckets)
    assert offs[0] == 0 and all(o % 256 == 0 for o in offs)
    assert all(b - a >= n for a, b, n in zip(offs, offs[1:], sizes))
    total = offs[-1] + (sizes[-1] + 255) // 256 * 256
    assert 1 <= len(spans) <= buckets
    assert spans[0][0] == 0 and spans[-1][1] == total and spans[0][2] == 0 and spans[-1][3] == len(sizes)
    for (lo, hi, a, b), nxt in zip(spans, spans[1:] + [None]):
        assert lo == offs[a] and a < b and (hi == offs[b] if b < len(sizes) else hi == total)
        if nxt is not None:
            assert nxt[0] == hi and nxt[2] == b


def test_one_wave_share():
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    for members in (1, 2, 8, 51, 176, 2000):
        gx = rt.one_wave_share(members)
        assert gx >= 1 and (gx - 1) * members < cg.SM_COUNT * 8 <= gx * members or gx == 1
