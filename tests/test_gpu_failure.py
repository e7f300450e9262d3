"""Failure detection on the GPU without a GPU fault: a bounded wait that runs out.

A kernel waits on an mbarrier that nothing ever arrives on (the same bounded wait the tensor-core
GEMM uses, here with a 50 ms limit).  It must give up, record an error code in its error word and
return; the host reads the status, and the context stays usable for the next launch."""
import importlib
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SRC = r"""
#define TCB_WAIT_NS 50000000u
#include "tcb/common.cuh"
#define TCB_M 1
#define TCB_N 1
#define TCB_K 32
#define TCB_KP 32
#define TCB_BATCH 1
#define TCB_IA 0
#define TCB_IB 1
#define TCB_BN 128
#define TCB_STAGES 2
#define TCB_PART_OFFSET 0
struct Epi { __device__ static float apply(const tcb::Args&, float acc, u64, u64, u64, u64) { return acc; } };
#include "tcb/gemm_tc.cuh"
extern "C" __global__ void never_arrives(const tcb::Args a) {
  __shared__ __align__(8) unsigned long long bar;
  const u32 b = tcb::smem_u32(&bar);
  if (threadIdx.x == 0) tcb::mbar_init(b, 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = tcb::mbar_wait(b, 0, reinterpret_cast<u32*>(a.p[15]), 7);
    reinterpret_cast<float*>(a.out)[0] = ok ? 1.0f : -1.0f;
  }
}
extern "C" __global__ void runs_for(const tcb::Args a) {
  const unsigned long long t0 = tcb::now_ns();
  while (tcb::now_ns() - t0 < (unsigned long long)a.p[0]) { }
  if (threadIdx.x == 0) reinterpret_cast<float*>(a.out)[0] = 3.0f;
}
extern "C" __global__ void still_works(const tcb::Args a) {
  reinterpret_cast<float*>(a.out)[threadIdx.x] = 2.0f * threadIdx.x;
}
"""


def test_a_wait_that_never_completes_returns_an_error_status(pkg, runner):
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    mod = runner.pipeline(SRC)
    out = rt.DeviceBuffer(runner, 1024)
    err = rt.DeviceBuffer(runner, 16)
    try:
        err.upload(np.zeros(4, np.uint32))
        args = rt.make_args([], out.ptr, 0, [0] * 15 + [err.ptr])
        t0 = time.time()
        rt.check(rt.lib().tc_launch(mod.handle, b"never_arrives", rt._u32x3((1, 1, 1)), rt._u32x3((32, 1, 1)), 0,
                                    rt.ctypes.byref(args)))
        runner.sync(timeout_ms=10000)
        assert time.time() - t0 < 5
        assert err.download(1, np.uint32)[0] == 7          # the wait's own code
        assert out.download(1)[0] == -1.0                  # the kernel saw the wait fail and returned
        # the context is still usable
        rt.check(rt.lib().tc_launch(mod.handle, b"still_works", rt._u32x3((1, 1, 1)), rt._u32x3((64, 1, 1)), 0,
                                    rt.ctypes.byref(args)))
        runner.sync()
        assert np.array_equal(out.download(64), 2.0 * np.arange(64, dtype=np.float32))
    finally:
        out.free()
        err.free()


def test_host_sync_times_out_on_a_slow_kernel_and_recovers(pkg, runner):
    """The host's bounded wait (tc_sync) gives up on a kernel still running and returns TIMEOUT;
    the kernel (which always ends: it runs for a fixed 300 ms of %globaltimer) then completes
    and a later wait succeeds."""
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    mod = runner.pipeline(SRC)
    out = rt.DeviceBuffer(runner, 1024)
    try:
        args = rt.make_args([], out.ptr, 0, [300_000_000])
        rt.check(rt.lib().tc_launch(mod.handle, b"runs_for", rt._u32x3((1, 1, 1)), rt._u32x3((32, 1, 1)), 0,
                                    rt.ctypes.byref(args)))
        with pytest.raises(rt.TcError) as e:
            runner.sync(timeout_ms=20)
        assert e.value.status == 5                         # TC_ERR_TIMEOUT
        runner.sync(timeout_ms=10000)
        assert out.download(1)[0] == 3.0
    finally:
        out.free()
