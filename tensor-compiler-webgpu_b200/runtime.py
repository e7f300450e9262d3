"""The host runtime over libtcb200's C ABI: the replacement of the reference's src/gpu runtime.

* ``GpuRunner``  -- src/gpu/runtime.js:16-130: ``create``, ``info``,
  ``pipeline(code)`` (compiled once per source text), ``run(graph, lowered,
  inputs, canary)`` with a buffer per node, optional canary padding and every
  node read back.
* ``run_local``  -- src/gpu/harness-m3b.js:86: each launch reads
  float32-rounded reference operands and writes its own output.
* ``Program``    -- a lowered graph made resident: one arena planned from
  buffer lifetimes, every launch resolved into a native plan (tc_plan) that
  replays without host work or as one CUDA graph.
* ``GpuTrainer`` / ``FusedTrainer`` -- src/gpu/trainer.js:13-104 and
  src/fusion/trainer-fused.js:18-109: the persistent training step; each step
  writes x and y, runs every launch, copies every new parameter and state
  value into its input buffer on the device, and reads back the loss.

There is no CPU fallback: without the library or a B200 these raise.
"""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np

from . import build as _build
from .ir import size
from .codegen import lower, lower_fused, WG, KernelCall

TC_OK = 0
STATUS = {0: "OK", 1: "INVALID", 2: "CUDA", 3: "COMPILE", 4: "OOM", 5: "TIMEOUT", 6: "NCCL", 7: "UNAVAILABLE"}
SYNC_TIMEOUT_MS = int(os.environ.get("TCB_SYNC_TIMEOUT_MS", "120000"))


class TcError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class Args(ctypes.Structure):
    _fields_ = [("in_", ctypes.c_uint64 * 8), ("out", ctypes.c_uint64), ("scratch", ctypes.c_uint64),
                ("p", ctypes.c_int64 * 16)]


_lib = None

_SIGS = {
    "tc_last_error": ([], ctypes.c_char_p),
    "tc_version": ([], ctypes.c_int),
    "tc_templates_hash": ([], ctypes.c_uint64),
    "tc_open": ([ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "tc_close": ([ctypes.c_void_p], ctypes.c_int),
    "tc_info": ([ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "tc_get_stream": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "tc_set_stream": ([ctypes.c_void_p, ctypes.c_uint64], ctypes.c_int),
    "tc_alloc": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "tc_free": ([ctypes.c_void_p], ctypes.c_int),
    "tc_buf_ptr": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "tc_upload": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "tc_download": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "tc_check_canary": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "tc_memcpy_htod": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64], ctypes.c_int),
    "tc_memcpy_dtoh": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "tc_memcpy_dtod": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "tc_memset32": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64], ctypes.c_int),
    "tc_host_alloc": ([ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "tc_host_free": ([ctypes.c_void_p], ctypes.c_int),
    "tc_compile": ([ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p,
                    ctypes.c_size_t], ctypes.c_int),
    "tc_compile_check": ([ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64)],
                         ctypes.c_int),
    "tc_compile_cubin": ([ctypes.c_char_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64),
                          ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "tc_module_load": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)],
                       ctypes.c_int),
    "tc_module_free": ([ctypes.c_void_p], ctypes.c_int),
    "tc_launch": ([ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32),
                   ctypes.c_uint32, ctypes.POINTER(Args)], ctypes.c_int),
    "tc_launch_tma": ([ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32),
                       ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint32, ctypes.c_int, ctypes.POINTER(ctypes.c_uint64),
                       ctypes.POINTER(Args)], ctypes.c_int),
    "tc_sync": ([ctypes.c_void_p, ctypes.c_int], ctypes.c_int),
    "tc_stream_create": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "tc_stream_destroy": ([ctypes.c_void_p, ctypes.c_uint64], ctypes.c_int),
    "tc_memcpy_htod_on": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64],
                          ctypes.c_int),
    "tc_memcpy_dtoh_on": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64],
                          ctypes.c_int),
    "tc_event_record_on": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "tc_stream_wait_event": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "tc_event_sync": ([ctypes.c_uint64, ctypes.c_int], ctypes.c_int),
    "tc_plan_run_on": ([ctypes.c_void_p, ctypes.c_uint64], ctypes.c_int),
    "tc_event_create": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "tc_event_record": ([ctypes.c_void_p, ctypes.c_uint64], ctypes.c_int),
    "tc_event_elapsed_ms": ([ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(ctypes.c_float)], ctypes.c_int),
    "tc_event_destroy": ([ctypes.c_uint64], ctypes.c_int),
    "tc_plan_create": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "tc_plan_add_launch": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32),
                            ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint32, ctypes.POINTER(Args)], ctypes.c_int),
    "tc_plan_add_launch_tma": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32),
                                ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint32, ctypes.c_int,
                                ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(Args)], ctypes.c_int),
    "tc_plan_add_copy": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "tc_plan_add_allreduce": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float],
                              ctypes.c_int),
    "tc_plan_run": ([ctypes.c_void_p], ctypes.c_int),
    "tc_plan_capture": ([ctypes.c_void_p], ctypes.c_int),
    "tc_plan_launch_count": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "tc_plan_free": ([ctypes.c_void_p], ctypes.c_int),
    "tc_plan_memory": ([ctypes.c_int, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_int32),
                        ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_uint64),
                        ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "tc_colsum_f32_static": ([ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64],
                             ctypes.c_int),
    "tc_lower_json": ([ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "tc_lowered_count": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "tc_lowered_json": ([ctypes.c_void_p, ctypes.c_char_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "tc_lowered_free": ([ctypes.c_void_p], ctypes.c_int),
    "tc_lowered_run": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                        ctypes.c_int, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "tc_program_create": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                           ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)],
                          ctypes.c_int),
    "tc_program_write": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64], ctypes.c_int),
    "tc_program_read": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64], ctypes.c_int),
    "tc_program_run": ([ctypes.c_void_p], ctypes.c_int),
    "tc_program_check": ([ctypes.c_void_p], ctypes.c_int),
    "tc_program_ptr": ([ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "tc_program_launch_count": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "tc_program_free": ([ctypes.c_void_p], ctypes.c_int),
    "tc_comm_unique_id": ([ctypes.c_char_p], ctypes.c_int),
    "tc_comm_init": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                      ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "tc_allreduce_f32": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float], ctypes.c_int),
    "tc_allreduce_f32_on": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, ctypes.c_uint64],
                            ctypes.c_int),
    "tc_comm_wait": ([ctypes.c_void_p, ctypes.c_int], ctypes.c_int),
    "tc_comm_abort": ([ctypes.c_void_p], ctypes.c_int),
    "tc_comm_destroy": ([ctypes.c_void_p], ctypes.c_int),
}

EXPORTS = tuple(_SIGS)


def lib():
    """The loaded libtcb200.so (built in-tree if missing).  Raises if it cannot be built or loaded."""
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            _build.build()
        handle = ctypes.CDLL(path)
        for name, (argtypes, restype) in _SIGS.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = handle
    return _lib


def check(status):
    if status != TC_OK:
        raise TcError(status, lib().tc_last_error().decode(errors="replace"))


def _u32x3(v):
    return (ctypes.c_uint32 * 3)(*v)


def compile_check(code):
    """NVRTC-compile `code` for sm_100a without a device; returns the cubin size."""
    log = ctypes.create_string_buffer(1 << 16)
    nbytes = ctypes.c_uint64(0)
    st = lib().tc_compile_check(code.encode(), log, len(log), ctypes.byref(nbytes))
    if st != TC_OK:
        raise TcError(st, lib().tc_last_error().decode(errors="replace"))
    return nbytes.value


CACHE_DIR = os.environ.get("TCB_KERNEL_CACHE", os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                               "_kernel_cache"))


def _cache_path(code):
    """Cache file of a kernel: keyed by its source AND the library's embedded template text."""
    import hashlib
    key = hashlib.sha256(code.encode() + b"\0" + str(lib().tc_templates_hash()).encode()).hexdigest()[:32]
    return os.path.join(CACHE_DIR, key + ".cubin")


def compile_cubin(code):
    """NVRTC cubin for `code` (sm_100a), from the on-disk kernel cache when present; no device needed."""
    path = _cache_path(code)
    if os.path.exists(path):
        with open(path, "rb") as f:
            return f.read()
    n = ctypes.c_uint64(0)
    log = ctypes.create_string_buffer(1 << 16)
    check(lib().tc_compile_cubin(code.encode(), None, 0, ctypes.byref(n), log, len(log)))
    buf = ctypes.create_string_buffer(n.value)
    check(lib().tc_compile_cubin(code.encode(), buf, n.value, ctypes.byref(n), log, len(log)))
    data = buf.raw[:n.value]
    try:
        os.makedirs(CACHE_DIR, exist_ok=True)
        tmp = f"{path}.{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    except OSError:
        pass
    return data


def precompile(codes, threads=None):
    """Compile many sources in parallel threads into the kernel cache (ctypes releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor
    todo = sorted({c for c in codes if not os.path.exists(_cache_path(c))})
    if not todo:
        return 0
    with ThreadPoolExecutor(threads or min(16, os.cpu_count() or 4)) as ex:
        list(ex.map(compile_cubin, todo))
    return len(todo)


class Module:
    __slots__ = ("handle", "runner")

    def __init__(self, handle, runner):
        self.handle = handle
        self.runner = runner


def _map_desc(call, scratch, ins=(), out=0):
    """The 8-value tensor-map descriptors of a call (include/tcb200.h, tc_launch_tma): each map is over
    scratch (at an offset), one of the launch's operands ('in', operand index) or its output ('out')."""
    vals = []
    for region, off, cols, rows, batches, rs, bs, bc, br in call.tma:
        if region == "scratch":
            addr = scratch + off
        elif region == "in":
            addr = ins[off]
        elif region == "out":
            addr = out + off
        elif region == "abs":
            addr = off
        else:
            raise ValueError(f"tensor map over '{region}'")
        if addr % 16:
            raise ValueError(f"{call.name}: tensor map base {addr:#x} is not 16-byte aligned")
        vals += [addr, cols, rows, batches, rs, bs, bc, br]
    return (ctypes.c_uint64 * len(vals))(*vals)


def issue(call, mod, ins, out, scratch, plan=None, err_ptr=None, ptrs=None):
    """Launch one KernelCall now (plan None) or append it to a native plan.

    A call with an error word gets its address in p[15]: `err_ptr` when given (a resident program's own
    word for that launch), else its slot in the scratch buffer.  `ptrs` (node id -> device address)
    resolves a call's `out_node` and `ptr_params` (a launch with a second output).
    """
    params = list(call.params)
    if call.out_node is not None:
        out = ptrs[call.out_node]
    for k, nid in call.ptr_params:
        while len(params) <= k:
            params.append(0)
        params[k] = ptrs[nid]
    if call.err_offset is not None:
        while len(params) < 16:
            params.append(0)
        params[15] = err_ptr if err_ptr is not None else scratch + call.err_offset
    args = make_args(ins, out, scratch, params)
    g, b = _u32x3(call.grid), _u32x3(call.block)
    if call.tma:
        desc = _map_desc(call, scratch, ins, out)
        if plan is None:
            check(lib().tc_launch_tma(mod.handle, call.name.encode(), g, b, call.smem, len(call.tma), desc,
                                      ctypes.byref(args)))
        else:
            check(lib().tc_plan_add_launch_tma(plan, mod.handle, call.name.encode(), g, b, call.smem, len(call.tma),
                                               desc, ctypes.byref(args)))
    elif plan is None:
        check(lib().tc_launch(mod.handle, call.name.encode(), g, b, call.smem, ctypes.byref(args)))
    else:
        check(lib().tc_plan_add_launch(plan, mod.handle, call.name.encode(), g, b, call.smem, ctypes.byref(args)))


def make_args(in_ptrs, out_ptr, scratch=0, params=()):
    a = Args()
    if len(in_ptrs) > 8:
        raise ValueError(f"{len(in_ptrs)} operands (at most 8)")
    for k, p in enumerate(in_ptrs):
        a.in_[k] = p
    a.out = out_ptr
    a.scratch = scratch
    for k, v in enumerate(params):
        a.p[k] = int(v)
    return a


class DeviceBuffer:
    """A device allocation owned by the library (tc_alloc)."""
    __slots__ = ("handle", "ptr", "nbytes", "runner")

    def __init__(self, runner, nbytes, canary_bytes=0):
        h = ctypes.c_void_p()
        check(lib().tc_alloc(runner.ctx, int(nbytes), int(canary_bytes), ctypes.byref(h)))
        p = ctypes.c_uint64()
        check(lib().tc_buf_ptr(h, ctypes.byref(p)))
        self.handle, self.ptr, self.nbytes, self.runner = h, p.value, int(nbytes), runner

    def upload(self, arr, offset=0):
        a = np.ascontiguousarray(arr)
        check(lib().tc_upload(self.handle, a.ctypes.data, a.nbytes, offset))

    def download(self, count, dtype=np.float32, offset=0):
        out = np.empty(count, dtype=dtype)
        if out.nbytes:
            check(lib().tc_download(self.handle, out.ctypes.data, out.nbytes, offset))
        return out

    def canary_intact(self):
        ok = ctypes.c_int(1)
        check(lib().tc_check_canary(self.handle, ctypes.byref(ok)))
        return bool(ok.value)

    def free(self):
        if self.handle:
            check(lib().tc_free(self.handle))
            self.handle = None


class GpuRunner:
    """src/gpu/runtime.js's GpuRunner over libtcb200 (one device, one stream)."""

    def __init__(self, ctx, device):
        self.ctx = ctx
        self.device = device
        self.pipelines = {}
        self._scratch = None
        self.lost = None

    @staticmethod
    def create(device=0):
        h = ctypes.c_void_p()
        check(lib().tc_open(device, ctypes.byref(h)))
        return GpuRunner(h, device)

    def info(self):
        buf = ctypes.create_string_buffer(4096)
        check(lib().tc_info(self.ctx, buf, len(buf)))
        return json.loads(buf.value.decode())

    def pipeline(self, code):
        """The compiled module for `code`, built once (runtime.js:44-52)."""
        m = self.pipelines.get(code)
        if m is None:
            cubin = compile_cubin(code)
            h = ctypes.c_void_p()
            check(lib().tc_module_load(self.ctx, cubin, len(cubin), ctypes.byref(h)))
            m = self.pipelines[code] = Module(h, self)
        return m

    def scratch(self, nbytes):
        if nbytes <= 0:
            return 0
        if self._scratch is None or self._scratch.nbytes < nbytes:
            if self._scratch is not None:
                self.sync()
                self._scratch.free()
            self._scratch = DeviceBuffer(self, nbytes)
            check(lib().tc_memset32(self.ctx, self._scratch.ptr, 0, nbytes // 4))  # error words start clear
        return self._scratch.ptr

    def check_errors(self, lau, scratch):
        """A kernel's bounded wait that ran out leaves a nonzero error word: raise it (after a sync)."""
        for call in lau.calls:
            if call.err_offset is not None:
                w = np.zeros(1, np.uint32)
                check(lib().tc_memcpy_dtoh(self.ctx, w.ctypes.data, scratch + call.err_offset, 4))
                self.sync()
                if w[0]:
                    check(lib().tc_memset32(self.ctx, scratch + call.err_offset, 0, 1))
                    raise TcError(5, f"{call.name}: a bounded wait ran out (code {int(w[0])})")

    def stream(self):
        s = ctypes.c_uint64()
        check(lib().tc_get_stream(self.ctx, ctypes.byref(s)))
        return s.value

    def set_stream(self, handle):
        check(lib().tc_set_stream(self.ctx, int(handle)))

    def sync(self, timeout_ms=SYNC_TIMEOUT_MS):
        check(lib().tc_sync(self.ctx, int(timeout_ms)))

    def launch(self, lau, in_ptrs, out_ptr, ptrs=None):
        """Issue every kernel call of one Launch (asynchronous); `ptrs` maps node ids to device addresses
        for a launch with a second output."""
        mod = self.pipeline(lau.code)
        scratch = self.scratch(lau.scratch_bytes)
        for call in lau.calls:
            issue(call, mod, in_ptrs, out_ptr, scratch, ptrs=ptrs)
        return scratch

    def run(self, graph, lowered, inputs, canary=False):
        """Run `lowered` for `graph`; every node read back (runtime.js:60-129).

        Returns {"values": [float32 arrays per node], "canaryIntact": [bool per node] (with canary)}.
        """
        if self.lost:
            raise TcError(2, f"device lost: {self.lost}")
        bufs = []
        try:
            for node in graph.nodes:
                n = size(node.shape)
                pad = ((-(-n // WG)) * WG + WG - n) * 4 if canary else 0
                bufs.append(DeviceBuffer(self, max(1, n) * 4, pad))
            for node in graph.nodes:
                if node.op == "input":
                    v = np.asarray(inputs[node.attrs["name"]], dtype=np.float32).reshape(-1)
                    if v.size != size(node.shape):
                        raise ValueError(f"input '{node.attrs['name']}': expected {size(node.shape)} numbers, got {v.size}")
                    bufs[node.id].upload(v)
                elif node.op == "const":
                    v = node.attrs["value"]
                    arr = np.full(size(node.shape), v, dtype=np.float32) if isinstance(v, (int, float)) \
                        else np.asarray(v, dtype=np.float32)
                    bufs[node.id].upload(arr)
            checks = []
            ptrs = {node.id: bufs[node.id].ptr for node in graph.nodes}
            for lau in lowered["launches"]:
                sc = self.launch(lau, [bufs[i].ptr for i in lau.inputs], bufs[lau.node].ptr, ptrs)
                if any(c.err_offset is not None for c in lau.calls):
                    self.sync()
                    self.check_errors(lau, sc)
            self.sync()
            values = [bufs[node.id].download(size(node.shape)) for node in graph.nodes]
            intact = [b.canary_intact() for b in bufs] if canary else []
            return {"values": values, "canaryIntact": intact}
        finally:
            for b in bufs:
                b.free()

    def close(self):
        if self._scratch is not None:
            self._scratch.free()
            self._scratch = None
        if self.ctx:
            check(lib().tc_close(self.ctx))
            self.ctx = None


def run_local(runner, graph, lowered, values, canary=False):
    """Node-local run (src/gpu/harness-m3b.js:86): each launch on float32 reference operands.

    `values` are reference values per node (any float dtype); each launch's
    operands are uploaded rounded to float32, and its own output is read back.
    Returns a list with the output of every launched node (None elsewhere).
    """
    out = [None] * len(graph.nodes)
    for lau in lowered["launches"]:
        bufs = []
        try:
            ins = []
            for i in lau.inputs:
                b = DeviceBuffer(runner, max(1, size(graph.nodes[i].shape)) * 4)
                b.upload(np.asarray(values[i], dtype=np.float32).reshape(-1))
                bufs.append(b)
                ins.append(b.ptr)
            n = size(graph.nodes[lau.node].shape)
            ob = DeviceBuffer(runner, max(1, n) * 4, ((-(-n // WG)) * WG + WG - n) * 4 if canary else 0)
            bufs.append(ob)
            sc = runner.launch(lau, ins, ob.ptr)
            runner.sync()
            runner.check_errors(lau, sc)
            out[lau.node] = ob.download(n)
            if canary and not ob.canary_intact():
                raise TcError(1, f"launch for node {lau.node} wrote past its output")
        finally:
            for b in bufs:
                b.free()
    return out


def plan_memory(sizes, first, last):
    """Arena offsets for buffers with lifetimes [first, last] (tc_plan_memory: best fit, 256-byte aligned)."""
    n = len(sizes)
    b = (ctypes.c_uint64 * max(1, n))(*sizes)
    f = (ctypes.c_int32 * max(1, n))(*first)
    l_ = (ctypes.c_int32 * max(1, n))(*last)
    off = (ctypes.c_uint64 * max(1, n))()
    total = ctypes.c_uint64()
    check(lib().tc_plan_memory(n, b, f, l_, off, ctypes.byref(total)))
    return [off[i] for i in range(n)], total.value


BATCH_MAX_ELEMS = 1 << 20   # elementwise launches up to this many elements may be batched


class MultiLaunch:
    """Same-source elementwise launches over different buffers issued as one `tcb_elementwise_multi`
    launch (instance = blockIdx.y, argument blocks in a device table).  Stands at its last member's
    position in a program's launch order."""

    def __init__(self, members):
        self.members = members
        m0 = members[0]
        self.code = m0.code
        self.kind = "multi " + (m0.pattern or m0.kind)
        self.pattern = m0.pattern
        self.node = members[-1].node
        self.nodes = [m.node for m in members]
        self.inputs = [i for m in members for i in m.inputs]
        self.scratch_bytes = 0
        self.bytes = sum(m.bytes for m in members)
        self.info = {"members": len(members)}
        c = m0.calls[0]
        # the grid-stride loop covers every member's count: about one wave of CTAs over all members
        gx = min(max(m.calls[0].grid[0] for m in members), one_wave_share(len(members)))
        self.calls = [KernelCall("tcb_elementwise_multi", (gx, len(members), 1), c.block, c.smem, c.params)]


def one_wave_share(members, ctas_per_sm=8):
    """x-extent of a (gx, members) grid whose members each grid-stride over their own work: about one
    wave of CTAs in all.  Sizing every member for the largest one's count made tens of thousands of
    CTAs, most exiting at once (C5's weight split: 56 us for 13 MB)."""
    from .codegen import SM_COUNT
    return max(1, -(-SM_COUNT * ctas_per_sm // max(1, members)))


def batch_small_launches(launches, root, max_elems=BATCH_MAX_ELEMS):
    """Hoist small elementwise launches and batch the independent ones of one source.

    Every small launch (a single tcb_elementwise call, no scratch, at most `max_elems` elements) moves
    up to just after the launch that produces its last input: its slot is (anchor, depth), the anchor
    being the last large producer among its inputs' producers and the depth one more than the deepest
    small producer on that anchor.  Other launches keep their place, and moving a producer earlier
    never puts it after a reader, so the order stays a valid one.  Small launches of one source that
    land on the same slot cannot read one another (a reader is always deeper than what it reads) and
    run as one MultiLaunch there.  Only small values live longer, so the arena grows little."""
    def eligible(lau):
        return (len(lau.calls) == 1 and lau.calls[0].name == "tcb_elementwise" and not lau.scratch_bytes
                and lau.calls[0].err_offset is None and lau.calls[0].params and lau.calls[0].params[0] <= max_elems)
    producer = {}
    slot = []
    for k, lau in enumerate(launches):
        if eligible(lau):
            best = (-1, 0)
            for i in lau.inputs:
                p = producer.get(root(i))
                if p is not None:
                    cand = (slot[p][0], slot[p][1] + 1) if slot[p][1] > 0 else (p, 1)
                    best = max(best, cand)
            if best[1] == 0:
                best = (-1, 1)
            slot.append(best)
        else:
            slot.append((k, 0))
        for nid in getattr(lau, "nodes", None) or [lau.node]:   # a two-output launch produces both
            producer[nid] = k
    groups = {}
    for k, lau in enumerate(launches):
        if slot[k][1] > 0:
            groups.setdefault((slot[k], lau.code), []).append(k)
    rep = {}
    for members in groups.values():
        if len(members) > 1:
            rep[members[0]] = MultiLaunch([launches[k] for k in members])
            for k in members[1:]:
                rep[k] = None
    order = sorted(range(len(launches)), key=lambda k: (slot[k], k))
    out = []
    for k in order:
        if k in rep:
            if rep[k] is not None:
                out.append(rep[k])
        else:
            out.append(launches[k])
    return out


def select_launches(graph, lowered, keep=(), feedback=(), place=(), alias=True, batch=False, prune=True):
    """The launches a resident program over `lowered` issues, in order (Program's `prune`, `alias` and
    `batch` rules), with the alias map (reshape node -> its source) and the number pruned.  A pure
    function of its arguments: a caller that lays out memory by launch order (the data-parallel
    trainer's bucketed gradient buffer) gets the order the program will have."""
    nodes = graph.nodes
    keep = set(keep)
    place = set(place)
    fb = {i for pair in feedback for i in pair}
    amap = {}
    out = []
    live = None
    if prune:
        live = set(keep) | {src for src, _ in feedback} | place
        for n in reversed(nodes):
            if n.id in live:
                live.update(n.inputs)
    pruned = 0
    for lau in lowered["launches"]:
        if live is not None and not any(n in live for n in getattr(lau, "nodes", [lau.node])):
            pruned += 1
            continue
        n = nodes[lau.node]
        if (alias and n.op == "reshape" and lau.kind == "gather" and lau.node not in keep
                and lau.node not in place and lau.node not in fb):
            amap[lau.node] = lau.inputs[0]
            continue
        out.append(lau)

    def root(i):
        while i in amap:
            i = amap[i]
        return i
    if batch:
        out = batch_small_launches(out, root)
    return out, amap, pruned


class Program:
    """A lowered graph made resident on the device, replayed by a native plan.

    Inputs, constants and `keep` nodes get buffers of their own for the
    program's life; every other value lives in one arena at an offset planned
    from its lifetime (producing launch to last consuming launch), so peak
    memory is the live set, not the graph.  `feedback` pairs (from, to) append
    device copies after the last launch (the trainers' parameter/state
    feedback, src/gpu/trainer.js:64).
    """

    def __init__(self, runner, graph, lowered, keep=(), feedback=(), capture=False, place=None, alias=True,
                 batch=False, prune=True, collectives=()):
        """`place` maps node ids to device addresses owned by the caller (e.g. slices of one flat buffer).

        `collectives`: (node ids, device address, float count, scale, communicator handle) tuples -- a
        sum-allreduce of that range, issued on the plan's collective stream right after the last launch
        that writes any of those nodes, so the launches after it compute while it runs
        (tc_plan_add_allreduce); the plan's end waits for all of them.

        `prune`: launches whose values nothing reads -- no kept, fed-back or caller-placed value depends
        on them (autodiff's branches toward constants, say) -- are left out; every value the program
        exposes is unchanged.

        `alias`: a plain reshape launch is dropped and its value shares its source's memory (a row-major
        reshape moves no bytes); lifetimes are merged along alias chains.
        `batch`: small independent launches of one elementwise source run as one launch
        (`batch_small_launches`); values are unchanged, the number of launches drops.
        """
        self.runner = runner
        self.graph = graph
        nodes = graph.nodes
        self.own = {}
        keep = set(keep)
        place = place or {}
        fb = {i for pair in feedback for i in pair}
        launches, self.alias, self.pruned = select_launches(graph, lowered, keep, feedback, place, alias, batch, prune)

        def root(i):
            while i in self.alias:
                i = self.alias[i]
            return i
        self.launches = launches
        first, last = {}, {}
        for k, lau in enumerate(self.launches):
            for nid in getattr(lau, "nodes", [lau.node]):
                first[nid] = k
            for i in lau.inputs:
                r = root(i)
                last[r] = max(last.get(r, -1), k)
        consumed = set(last)
        arena_ids = []
        for node in nodes:
            nbytes = max(1, size(node.shape)) * 4
            if node.id in place or node.id in self.alias:
                continue
            if node.op in ("input", "const") or node.id in keep or node.id in fb:
                self.own[node.id] = DeviceBuffer(runner, nbytes)
            elif node.id in first:
                arena_ids.append(node.id)
            elif node.id in consumed:
                self.own[node.id] = DeviceBuffer(runner, nbytes)
            # else: never produced nor read (a folded transpose): no memory
        offs, total = plan_memory([max(1, size(nodes[i].shape)) * 4 for i in arena_ids],
                                  [first[i] for i in arena_ids], [last.get(i, first[i]) for i in arena_ids])
        self.arena_bytes = total
        self.arena = DeviceBuffer(runner, max(total, 256)) if arena_ids else None
        self.ptrs = {i: b.ptr for i, b in self.own.items()}
        self.ptrs.update(place)
        for i, o in zip(arena_ids, offs):
            self.ptrs[i] = self.arena.ptr + o
        for a in self.alias:
            self.ptrs[a] = self.ptrs[root(a)]
        for node in nodes:
            if node.op == "const" and node.id in self.own:
                v = node.attrs["value"]
                arr = np.full(size(node.shape), v, dtype=np.float32) if isinstance(v, (int, float)) \
                    else np.asarray(v, dtype=np.float32)
                self.own[node.id].upload(arr)
        scratch_bytes = max([lau.scratch_bytes for lau in self.launches] + [0])
        self.scratch = DeviceBuffer(runner, scratch_bytes) if scratch_bytes else None
        if self.scratch:
            check(lib().tc_memset32(runner.ctx, self.scratch.ptr, 0, scratch_bytes // 4))
        # a private control block (error word + split-tile arrival counters) per launch that has one:
        # launches share scratch, so not there.  The blocks start zeroed and stay so -- a bounded wait
        # writes the error word only when it runs out (check_errors zeroes them again), the counters
        # return to zero as each split tile completes -- so the one-block clearing launch
        # (tcb_gemm_prep) that a one-off run needs is left out of the plan.
        self.err_slot = {}
        off = 0
        for k, lau in enumerate(self.launches):
            if any(c.err_offset is not None for c in lau.calls):
                self.err_slot[k] = off
                off += (lau.info or {}).get("ctrl_bytes", 64)
        self.errs_bytes = max(64, off)
        self.errs = DeviceBuffer(runner, self.errs_bytes)
        check(lib().tc_memset32(runner.ctx, self.errs.ptr, 0, self.errs_bytes // 4))
        h = ctypes.c_void_p()
        check(lib().tc_plan_create(runner.ctx, ctypes.byref(h)))
        self.plan = h
        self.kernel_launches = 0
        self.tables = []
        self.split_bufs = []
        self.hoisted = {}
        self._hoist = None
        if batch:
            self.kernel_launches += self._hoist_input_splits(h)
        done_at = {}
        for k, lau in enumerate(self.launches):
            for nid in getattr(lau, "nodes", [lau.node]):
                done_at[nid] = k
        after = {}
        for ids, ptr, count, scale, comm in collectives:
            after.setdefault(max(done_at[i] for i in ids), []).append((ptr, count, scale, comm))
        self.collectives = len(collectives)
        for k, lau in enumerate(self.launches):
            for call in program_calls(lau):
                if k in self.hoisted and call.name == "tcb_split_b":
                    continue
                self.issue_call(k, lau, call, h)
                self.kernel_launches += 1
            for ptr, count, scale, comm in after.get(k, ()):
                check(lib().tc_plan_add_allreduce(h, comm, ptr, count, ctypes.c_float(scale)))
        if batch and feedback:
            self.kernel_launches += self._issue_copies(feedback, h)
        else:
            for src, dst in feedback:
                check(lib().tc_plan_add_copy(h, self.ptrs[dst], self.ptrs[src], max(1, size(nodes[dst].shape)) * 4))
        self.captured = False
        if capture:
            self.capture()

    def _hoist_input_splits(self, plan):
        """Split every tensor-core launch's B operand that no launch of this program produces (a
        program input: the weights of a training step) in one tcb_split_multi launch at the start of
        the plan, into buffers of their own; those launches skip their split_b pass and their GEMM
        reads B_hi / B_lo there.  Returns the launches added (0 or 1)."""
        from .codegen import split_multi_source, grid1d
        produced = set()
        for lau in self.launches:
            produced.update(getattr(lau, "nodes", [lau.node]))
        jobs = []
        for k, lau in enumerate(self.launches):
            info = lau.info or {}
            if info.get("path") != "tcgen05-3xtf32" or not any(c.name == "tcb_split_b" for c in lau.calls):
                continue
            b_node = lau.inputs[info["ib"]]
            r = b_node
            while r in self.alias:
                r = self.alias[r]
            if r in produced:
                continue
            batch, M, K, N = info["mnk"]
            kp = info["kp"]
            nbytes = batch * N * kp * 4
            buf = DeviceBuffer(self.runner, 2 * nbytes)
            self.split_bufs.append(buf)
            self.hoisted[k] = (buf.ptr, buf.ptr + nbytes)
            jobs.append((self.ptrs[b_node], buf.ptr, buf.ptr + nbytes, batch, N, K, kp, 0 if info["b_t"] else 1))
        if not jobs:
            return 0
        table = (ctypes.c_uint64 * (8 * len(jobs)))(*[v for j in jobs for v in j])
        tbuf = DeviceBuffer(self.runner, ctypes.sizeof(table))
        check(lib().tc_upload(tbuf.handle, ctypes.addressof(table), ctypes.sizeof(table), 0))
        self.tables.append(tbuf)
        gx = 1
        for src, hi, lo, b, R, C, kp, cols in jobs:
            gx = max(gx, grid1d(b * R * kp, per_thread=1)[0] if not cols else min(b * (kp // 32) * -(-R // 32), 148 * 8))
        gx = min(gx, one_wave_share(len(jobs)))   # every job grid-strides: about one wave of CTAs in all
        mod = self.runner.pipeline(split_multi_source())
        self._hoist = (KernelCall("tcb_split_multi", (gx, len(jobs), 1), (256, 1, 1), 0, []), mod, tbuf.ptr)
        issue(self._hoist[0], mod, [], 0, tbuf.ptr, plan=plan)
        return 1

    def _issue_copies(self, feedback, plan):
        """The feedback copies as one multi-instance copy launch per vector width; returns the launches."""
        from .codegen import copy_source, grid1d
        by_w = {}
        for src, dst in feedback:
            n = max(1, size(self.graph.nodes[dst].shape))
            w = 4 if self.ptrs[src] % 16 == 0 and self.ptrs[dst] % 16 == 0 else 1
            by_w.setdefault(w, []).append((self.ptrs[src], self.ptrs[dst], n))
        for w, items in by_w.items():
            mod = self.runner.pipeline(copy_source(w))
            table = (Args * len(items))()
            for j, (a, b, n) in enumerate(items):
                table[j] = make_args([a], b, 0, [n])
            buf = DeviceBuffer(self.runner, ctypes.sizeof(table))
            check(lib().tc_upload(buf.handle, ctypes.addressof(table), ctypes.sizeof(table), 0))
            self.tables.append(buf)
            gx = min(max(grid1d(n, per_thread=w)[0] for _, _, n in items), one_wave_share(len(items)))
            issue(KernelCall("tcb_elementwise_multi", (gx, len(items), 1), (WG, 1, 1), 0, [0]), mod, [], 0, buf.ptr,
                  plan=plan)
        return len(by_w)

    def issue_call(self, k, lau, call, plan):
        """Append one kernel call of launch `k` to a native plan (a MultiLaunch gets its argument table)."""
        mod = self.runner.pipeline(lau.code)
        scratch = self.scratch.ptr if self.scratch else 0
        if isinstance(lau, MultiLaunch):
            table = (Args * len(lau.members))()
            for j, m in enumerate(lau.members):
                table[j] = make_args([self.ptrs[i] for i in m.inputs], self.ptrs[m.node], 0, m.calls[0].params)
            buf = DeviceBuffer(self.runner, ctypes.sizeof(table))
            check(lib().tc_upload(buf.handle, ctypes.addressof(table), ctypes.sizeof(table), 0))
            self.tables.append(buf)
            issue(call, mod, [], 0, buf.ptr, plan=plan)
            return
        if k in self.hoisted and call.tma:
            # this GEMM's B_hi / B_lo were split at the start of the plan into buffers of their own
            hi, lo = self.hoisted[k]
            tma = list(call.tma)
            tma[2] = ("abs", hi) + tuple(tma[2][2:])
            tma[3] = ("abs", lo) + tuple(tma[3][2:])
            orig = call
            call = KernelCall(orig.name, orig.grid, orig.block, orig.smem, orig.params)
            call.tma, call.err_offset = tma, orig.err_offset
        issue(call, mod, [self.ptrs[i] for i in lau.inputs], self.ptrs[lau.node], scratch, plan=plan,
              err_ptr=self.err_ptr(k), ptrs=self.ptrs)

    def capture(self):
        check(lib().tc_plan_capture(self.plan))
        self.captured = True

    def ptr(self, nid):
        return self.ptrs[nid]

    def write(self, nid, arr):
        """Synchronous upload into node `nid`'s buffer (float32)."""
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32).reshape(-1))
        if a.size != size(self.graph.nodes[nid].shape):
            raise ValueError(f"node {nid}: {a.size} values for shape {self.graph.nodes[nid].shape}")
        check(lib().tc_memcpy_htod(self.runner.ctx, self.ptrs[nid], a.ctypes.data, a.nbytes))
        self.runner.sync()

    def write_async(self, nid, host_ptr, nbytes):
        check(lib().tc_memcpy_htod(self.runner.ctx, self.ptrs[nid], host_ptr, nbytes))

    def read(self, nid):
        n = size(self.graph.nodes[nid].shape)
        out = np.empty(n, dtype=np.float32)
        self.runner.sync()
        if n:
            check(lib().tc_memcpy_dtoh(self.runner.ctx, out.ctypes.data, self.ptrs[nid], out.nbytes))
        self.runner.sync()
        return out

    def run(self):
        check(lib().tc_plan_run(self.plan))

    def err_ptr(self, k):
        return self.errs.ptr + self.err_slot[k] if k in self.err_slot else None

    def check_errors(self):
        """Raise if any tensor-core launch's bounded wait ran out (its own error word, read after a sync)."""
        if not self.err_slot:
            return
        self.runner.sync()
        w = self.errs.download(self.errs_bytes // 4, np.uint32)
        bad = [k for k, off in self.err_slot.items() if w[off // 4]]
        if bad:
            check(lib().tc_memset32(self.runner.ctx, self.errs.ptr, 0, self.errs_bytes // 4))
            raise TcError(5, f"launch {bad[0]} ({self.launches[bad[0]].kind}): a bounded wait ran out "
                             f"(code {int(w[self.err_slot[bad[0]] // 4])})")

    def free(self):
        if self.plan:
            check(lib().tc_plan_free(self.plan))
            self.plan = None
        for b in self.own.values():
            b.free()
        self.own = {}
        if self.arena:
            self.arena.free()
            self.arena = None
        if self.scratch:
            self.scratch.free()
            self.scratch = None
        for b in getattr(self, "tables", []) + getattr(self, "split_bufs", []):
            b.free()
        self.tables = []
        self.split_bufs = []
        if getattr(self, "errs", None):
            self.errs.free()
            self.errs = None


def fused_step(step, sabotage=None, pass_sabotage=None, matmul="naive"):
    """Fuse a step keeping the loss, logits and every output; ids renumbered (src/fusion/trainer-fused.js:18-29)."""
    from .fuse import fuse
    keep = [step["loss"], step["logits"], *step["outputs"].values()]
    f = fuse(step["graph"], keep=keep, sabotage=pass_sabotage)

    def at(i):
        return f.index[i]
    out = dict(step)
    out.update({"graph": f.graph, "fusion": f, "original": step["graph"], "loss": at(step["loss"]),
                "logits": at(step["logits"]),
                "inputs": {k: at(v) for k, v in step["inputs"].items()},
                "outputs": {k: at(v) for k, v in step["outputs"].items()},
                "lowered": lower_fused(f.graph, matmul=matmul, sabotage=sabotage)})
    if "cotangent" in step:
        out["cotangent"] = step["cotangent"]
    return out


class GpuTrainer:
    """The persistent training step (src/gpu/trainer.js:13-104; fused: src/fusion/trainer-fused.js:135-213).

    `step` is a builder result (steps.build_mlp_step / build_step3b) or a
    fused_step() of one.  Parameters and state stay on the device; each
    train() writes x and y, replays the step (one CUDA graph when `capture`),
    copies every new parameter/state value into its input and reads the loss.
    """

    def __init__(self, runner, step, params, state, matmul="naive", sabotage=None, capture=True, lowered=None):
        self.runner = runner
        self.step = step
        graph = step["graph"]
        if lowered is None:
            lowered = step.get("lowered") or lower(graph, matmul=matmul, sabotage=sabotage)
        names = list(params) + list(state)
        feedback = [(step["outputs"][n], step["inputs"][n]) for n in names]
        keep = {step["loss"], *[step["outputs"][n] for n in names]}
        self.prog = Program(runner, graph, lowered, keep=keep, feedback=feedback, batch=True)
        cot = graph.input_id(step["cotangent"])
        if cot is not None:
            self.prog.write(cot, [1.0])
        for n, v in {**params, **state}.items():
            self.prog.write(step["inputs"][n], v)
        if capture:
            self.prog.capture()

    def train(self, x, y):
        """One step on batch (x, y); returns the loss from the parameters before the update."""
        s = self.step
        self.prog.write(s["inputs"]["x"], x)
        self.prog.write(s["inputs"]["y"], y)
        self.prog.run()
        return float(self.prog.read(s["loss"])[0])

    def read(self, names):
        return {n: self.prog.read(self.step["inputs"][n]) for n in names}

    def destroy(self):
        self.prog.free()


class FusedTrainer(GpuTrainer):
    """GpuTrainer over a fused_step() (its lowering passed in, src/fusion/trainer-fused.js:135-161)."""

    def __init__(self, runner, step, params, state, capture=True):
        super().__init__(runner, step, params, state, capture=capture, lowered=step["lowered"])


def program_calls(lau):
    """The calls of a launch that a resident program issues: all but the control-block clearing."""
    return [c for c in lau.calls if c.name != "tcb_gemm_prep"]


class Segments:
    """Native plans over consecutive kernel-call ranges of a Program, so events can sit between them.

    `cuts` are indices into the flat list of kernel calls (every call of every launch, in order, as the
    program issues them: `program_calls`).
    """

    def __init__(self, prog, cuts):
        self.prog = prog
        self.plans = []
        flat = [(k, lau, call) for k, lau in enumerate(prog.launches) for call in program_calls(lau)
                if not (k in prog.hoisted and call.name == "tcb_split_b")]
        bounds = [0, *cuts, len(flat)]
        for a, b in zip(bounds[:-1], bounds[1:]):
            h = ctypes.c_void_p()
            check(lib().tc_plan_create(prog.runner.ctx, ctypes.byref(h)))
            if a == 0 and prog._hoist is not None:  # the program's up-front operand splits
                issue(prog._hoist[0], prog._hoist[1], [], 0, prog._hoist[2], plan=h)
            for k, lau, call in flat[a:b]:
                prog.issue_call(k, lau, call, h)
            self.plans.append(h)

    def run(self, k):
        check(lib().tc_plan_run(self.plans[k]))

    def free(self):
        for h in self.plans:
            check(lib().tc_plan_free(h))
        self.plans = []


class Events:
    """CUDA events on the runner's stream."""

    def __init__(self, runner, n):
        self.runner = runner
        self.ev = []
        for _ in range(n):
            e = ctypes.c_uint64()
            check(lib().tc_event_create(runner.ctx, ctypes.byref(e)))
            self.ev.append(e.value)

    def record(self, k):
        check(lib().tc_event_record(self.runner.ctx, self.ev[k]))

    def ms(self, a, b):
        v = ctypes.c_float()
        check(lib().tc_event_elapsed_ms(self.ev[a], self.ev[b], ctypes.byref(v)))
        return float(v.value)

    def free(self):
        for e in self.ev:
            check(lib().tc_event_destroy(e))
        self.ev = []


class PinnedHost:
    """Page-locked host memory (for the end-to-end path's copies)."""

    def __init__(self, nbytes):
        p = ctypes.c_void_p()
        check(lib().tc_host_alloc(int(max(1, nbytes)), ctypes.byref(p)))
        self.ptr = p.value
        self.nbytes = int(nbytes)

    def array(self, count, dtype=np.float32):
        buf = (ctypes.c_char * self.nbytes).from_address(self.ptr)
        return np.frombuffer(buf, dtype=dtype, count=count)

    def free(self):
        if self.ptr:
            check(lib().tc_host_free(self.ptr))
            self.ptr = None


class StreamedProgram:
    """A resident program fed from and drained to host memory, copies overlapped across steps.

    `slots` device copies of the program (inputs, arena, outputs) rotate; each `submit` copies one
    step's inputs in on an input stream, runs the program on the compute stream once they have
    landed, and copies its outputs out on an output stream -- so step k's outputs travel while step
    k+1's inputs travel the other way.  Every step still moves all of its own inputs and outputs.
    """

    def __init__(self, runner, graph, lowered, inputs, outputs, slots=2, capture=True):
        self.runner = runner
        self.inputs, self.outputs = list(inputs), list(outputs)
        self.progs = [Program(runner, graph, lowered, keep=outputs) for _ in range(slots)]
        if capture:
            for p in self.progs:
                p.capture()
        lib_ = lib()
        self.s_in, self.s_out = ctypes.c_uint64(), ctypes.c_uint64()
        check(lib_.tc_stream_create(runner.ctx, ctypes.byref(self.s_in)))
        check(lib_.tc_stream_create(runner.ctx, ctypes.byref(self.s_out)))
        self.s_in, self.s_out = self.s_in.value, self.s_out.value
        self.s_comp = runner.stream()
        self.ev = Events(runner, 3 * slots + 2)
        self.slots = slots
        self.used = [False] * slots
        self.k = 0

    def _rec(self, k, stream):
        check(lib().tc_event_record_on(self.runner.ctx, self.ev.ev[k], stream))

    def _wait(self, stream, k):
        check(lib().tc_stream_wait_event(self.runner.ctx, stream, self.ev.ev[k]))

    def mark(self, which):
        """Record timing event 0 ('start', on the input stream) or 1 ('end', on the output stream)."""
        k = 3 * self.slots + (0 if which == "start" else 1)
        self._rec(k, self.s_in if which == "start" else self.s_out)

    def elapsed_ms(self):
        return self.ev.ms(3 * self.slots, 3 * self.slots + 1)

    def submit(self, host_in, host_out):
        """host_in / host_out: {node id: (host pointer, bytes)} for every input and output."""
        S = self.slots
        slot = self.k % S
        p = self.progs[slot]
        IN, COMP, OUT = 3 * slot, 3 * slot + 1, 3 * slot + 2
        lib_ = lib()
        if self.used[slot]:
            self._wait(self.s_in, COMP)       # the slot's previous step has read its inputs
        for nid in self.inputs:
            ptr, n = host_in[nid]
            check(lib_.tc_memcpy_htod_on(self.runner.ctx, p.ptr(nid), ptr, n, self.s_in))
        self._rec(IN, self.s_in)
        self._wait(self.s_comp, IN)
        if self.used[slot]:
            self._wait(self.s_comp, OUT)      # ... and its outputs have left
        check(lib_.tc_plan_run_on(p.plan, self.s_comp))
        self._rec(COMP, self.s_comp)
        self._wait(self.s_out, COMP)
        for nid in self.outputs:
            ptr, n = host_out[nid]
            check(lib_.tc_memcpy_dtoh_on(self.runner.ctx, ptr, p.ptr(nid), n, self.s_out))
        self._rec(OUT, self.s_out)
        self.used[slot] = True
        self.k += 1

    def drain(self, timeout_ms=SYNC_TIMEOUT_MS):
        k = 3 * self.slots + 1
        self._rec(k, self.s_out)
        check(lib().tc_event_sync(self.ev.ev[k], timeout_ms))

    def free(self):
        self.drain()
        self.runner.sync()
        for p in self.progs:
            p.free()
        self.ev.free()
        check(lib().tc_stream_destroy(self.runner.ctx, self.s_in))
        check(lib().tc_stream_destroy(self.runner.ctx, self.s_out))
