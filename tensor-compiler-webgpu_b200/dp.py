"""Data-parallel training over the batch: one process per GPU, the gradients sum-allreduced over NCCL.

The step is split where the reference's step builder exposes the gradients
(src/m3b/step.js:18-31): a gradient graph (forward + loss + autodiff
backward) run on this rank's shard of the batch, then an Adam graph
(src/m3b/adam.js:24-48) run identically on every rank, so parameters stay
replicated.  Every gradient -- laid out back to back in one flat device buffer
that the gradient graph writes directly -- is sum-allreduced over
NVLink/NVSwitch and scaled by 1/W (each rank's loss divides by its local row
count, src/m3b/model.js:127-130, so the average of the rank gradients is the
full-batch gradient).  The buffer is ordered by when the backward finishes each
gradient and cut into a few contiguous buckets; each bucket's allreduce runs on
a collective stream while the rest of the backward computes, and the Adam graph
waits for all of them.  World size 1 skips the collective.

Process plumbing (rank, world, the NCCL unique id) goes through
torch.distributed's gloo group on the host; the collective itself is the
library's own tc_allreduce_f32 (NCCL, non-blocking communicator, bounded
waits).  No TMA, no multicast: remote data arrives only through NCCL.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from .codegen import lower_fused
from .fuse import fuse
from .ir import size
from . import runtime as rt
from . import steps as _steps

COMM_TIMEOUT_MS = 120000
DEFAULT_BUCKETS = 4


def bucket_layout(nbytes, buckets):
    """Offsets of tensors of `nbytes` laid out back to back in this order (256-byte aligned slices), and
    at most `buckets` contiguous spans (lo, hi, first index, end index) covering the whole layout, cut
    at tensor boundaries into about equal bytes: a tensor that starts in a later `buckets`-th of the
    total than the current span's first tensor opens a new span."""
    offs, total = [], 0
    for n in nbytes:
        offs.append(total)
        total += (n + 255) // 256 * 256
    spans, start = [], 0
    for j in range(1, len(offs) + 1):
        if j == len(offs) or offs[j] * buckets // max(total, 1) > offs[start] * buckets // max(total, 1):
            spans.append((offs[start], offs[j] if j < len(offs) else total, start, j))
            start = j
    return offs, spans


class Comm:
    """A libtcb200 NCCL communicator bootstrapped through a torch.distributed (gloo) group."""

    def __init__(self, runner, rank, world, timeout_ms=COMM_TIMEOUT_MS):
        import torch.distributed as dist
        lib = rt.lib()
        uid = ctypes.create_string_buffer(128)
        if rank == 0:
            rt.check(lib.tc_comm_unique_id(uid))
        box = [bytes(uid.raw) if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        uid = ctypes.create_string_buffer(box[0], 128)
        h = ctypes.c_void_p()
        rt.check(lib.tc_comm_init(runner.ctx, rank, world, uid, timeout_ms, ctypes.byref(h)))
        self.handle = h
        self.runner = runner
        self.rank, self.world = rank, world

    def allreduce_mean(self, ptr, count, prescaled=False):
        """Sum-allreduce, scaled by 1/W inside the collective (NCCL PreMulSum) unless the values were
        scaled already (`prescaled`: then a plain sum, which NCCL can also run as an NVLS reduction)."""
        scale = 1.0 if prescaled else 1.0 / self.world
        rt.check(rt.lib().tc_allreduce_f32(self.handle, ptr, count, ctypes.c_float(scale)))

    def wait(self, timeout_ms=COMM_TIMEOUT_MS):
        rt.check(rt.lib().tc_comm_wait(self.handle, timeout_ms))

    def destroy(self):
        if self.handle:
            rt.check(rt.lib().tc_comm_destroy(self.handle))
            self.handle = None


class DPTrainer:
    """The transformer training step, data parallel.  `batch_local` sequences per rank."""

    def __init__(self, runner, V, batch_local, cfg, params, state=None, comm=None, opt=_steps.ADAM_3B,
                 matmul="tiled", capture=True, batch=True, colfuse=True, mofuse=True, buckets=None):
        """`colfuse`: every bias gradient (a sum over axis 0) runs inside its elementwise producer's
        launch (codegen.colsum_fusions); `mofuse`: an elementwise reader runs in its producer's pass
        (codegen.mo_fusions).  Values are bitwise those of the separate launches either way.

        `buckets` (world > 1; default $TCB_DP_BUCKETS, else DEFAULT_BUCKETS): the flat gradient buffer
        is laid out in the order the backward finishes the gradients and cut into that many contiguous
        buckets of about equal bytes; each bucket's allreduce is issued on the collective stream as soon
        as its last gradient is written, so it runs while the rest of the backward computes.  1 = one
        allreduce of the whole buffer after the gradient program."""
        self.runner, self.comm = runner, comm
        gs = _steps.build_grad3b(V, batch_local, cfg)
        ad = _steps.build_adam_graph(V, cfg, opt)
        names = gs["names"]
        self.names = names
        shapes = _steps.param_shapes(V, cfg)
        # fused gradient graph: keep the loss and every gradient
        keep = [gs["loss"], *[gs["grads"][n] for n in names]]
        fg = fuse(gs["graph"], keep=keep)
        self.loss_id = fg.index[gs["loss"]]
        grad_ids = [fg.index[gs["grads"][n]] for n in names]
        lowered_g = lower_fused(fg.graph, matmul=matmul, fold=True, keep=[self.loss_id, *grad_ids], colfuse=colfuse,
                                mofuse=mofuse)
        self.lowered_g = lowered_g
        w = comm.world if comm is not None else 1
        if buckets is None:
            buckets = int(os.environ.get("TCB_DP_BUCKETS", DEFAULT_BUCKETS))
        self.buckets = max(1, buckets) if w > 1 else 1
        input_ids = [fg.index[gs["inputs"][n]] for n in names]
        order = list(range(len(names)))
        if self.buckets > 1:
            launches, _, _ = rt.select_launches(fg.graph, lowered_g, keep=[self.loss_id],
                                                place=set(input_ids) | set(grad_ids), batch=batch)
            done = {}
            for k, lau in enumerate(launches):
                for nid in getattr(lau, "nodes", [lau.node]):
                    done[nid] = k
            order.sort(key=lambda j: (done.get(grad_ids[j], -1), j))
        # one flat gradient buffer, each gradient at its offset (256-byte aligned slices)
        offs, spans = bucket_layout([size(shapes[names[j]]) * 4 for j in order], self.buckets)
        self.order = [names[j] for j in order]
        at = dict(zip(order, offs))
        offs = [at[j] for j in range(len(names))]
        total = spans[-1][1] if spans else 0
        self.flat = rt.DeviceBuffer(runner, max(total, 256))
        self.flat_floats = total // 4
        rt.check(rt.lib().tc_memset32(runner.ctx, self.flat.ptr, 0, max(total, 256) // 4))  # padding, zero grads
        # parameters: one buffer each, shared by both graphs (the Adam graph's outputs are copied back)
        self.params = {n: rt.DeviceBuffer(runner, size(shapes[n]) * 4) for n in names}
        place_g = {iid: self.params[n].ptr for iid, n in zip(input_ids, names)}
        # a gradient the graph gives as a constant zero (no dependence) is still written by its launch
        for gid, off in zip(grad_ids, offs):
            place_g[gid] = self.flat.ptr + off
        # With a power-of-two world the 1/W of the mean goes into the cotangent seed: backpropagation is
        # linear in it and a power-of-two scale is exact in every operation, so each rank's gradients
        # come out as exactly 1/W times its own, and the allreduce is a plain sum.
        self.prescaled = w > 1 and (w & (w - 1)) == 0
        colls = []
        self.bucket_spans = [(lo, hi) for lo, hi, _, _ in spans]
        if self.buckets > 1:
            scale = 1.0 if self.prescaled else 1.0 / w
            for lo, hi, a, b in spans:
                colls.append(([grad_ids[order[i]] for i in range(a, b)], self.flat.ptr + lo, (hi - lo) // 4, scale,
                              comm.handle))
        self.grad_prog = rt.Program(runner, fg.graph, lowered_g, keep=[self.loss_id], place=place_g, batch=batch,
                                    collectives=colls)
        fa = fuse(ad["graph"], keep=list(ad["outputs"].values()))
        place_a = {}
        for n, off in zip(names, offs):
            place_a[fa.index[ad["inputs"][f"g:{n}"]]] = self.flat.ptr + off
            place_a[fa.index[ad["inputs"][n]]] = self.params[n].ptr
        state_names = [k for k in ad["inputs"] if k not in names and not k.startswith("g:")]
        feedback = [(fa.index[ad["outputs"][n]], fa.index[ad["inputs"][n]]) for n in names + state_names]
        self.adam_prog = rt.Program(runner, fa.graph, lower_fused(fa.graph, matmul=matmul),
                                    keep=[fa.index[ad["outputs"][k]] for k in names + state_names],
                                    feedback=feedback, place=place_a, batch=batch)
        self.fa, self.ad, self.fg, self.gs = fa, ad, fg, gs
        self.state_names = state_names
        for n in names:
            self.params[n].upload(np.asarray(params[n], dtype=np.float32))
        if state is None:
            state = _steps.adam_initial_state(names, shapes)
        for k in state_names:
            self.adam_prog.write(fa.index[ad["inputs"][k]], state[k])
        cot = fg.graph.input_id(gs["cotangent"])
        self.grad_prog.write(cot, [1.0 / w if self.prescaled else 1.0])
        self.x_id = fg.index[gs["inputs"]["x"]]
        self.y_id = fg.index[gs["inputs"]["y"]]
        self.kernel_launches = self.grad_prog.kernel_launches + self.adam_prog.kernel_launches
        if capture:
            self.grad_prog.capture()
            self.adam_prog.capture()

    def step_device(self):
        """One step with x, y already on the device: gradients, allreduce, Adam (asynchronous)."""
        self.grad_prog.run()   # with buckets, the allreduces run inside it
        if self.comm is not None and self.comm.world > 1 and self.buckets == 1:
            self.comm.allreduce_mean(self.flat.ptr, self.flat_floats, prescaled=self.prescaled)
        self.adam_prog.run()

    def train(self, x, y):
        self.grad_prog.write(self.x_id, x)
        self.grad_prog.write(self.y_id, y)
        self.step_device()
        if self.comm is not None and self.comm.world > 1:
            self.comm.wait()
        return float(self.grad_prog.read(self.loss_id)[0])

    def read(self, names):
        self.runner.sync()
        return {n: self.params[n].download(self.params[n].nbytes // 4) for n in names}

    def destroy(self):
        self.grad_prog.free()
        self.adam_prog.free()
        self.flat.free()
        for b in self.params.values():
            b.free()
