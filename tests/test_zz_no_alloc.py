"""The allocation-free column sum (tc_colsum_f32_static) against the library's regular reduction.

tc_colsum_f32_static serves callers that cannot allocate device memory where
they need a column sum -- inside a stream capture, under another allocator's
fixed budget, or on a path that cannot take cudaMalloc's device-wide
synchronisation.  Its partial sums live in a static device array, so this test
checks that two calls in a row (the second finding the first call's partials
still in the array) both agree with the regular NVRTC `sum` over axis 0, whose
scratch the runner allocates.  Tolerance: the float32 budget -- each result is
within 2E of the exact float64 sum (E = gamma(rows) * sum |x|), so the two
agree within 4E.  This file sorts last so that a run stopping at its first
failure has already run every other test.
"""
import ctypes
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _regular_colsum(pkg, rt, cg, runner, x_buf, out_buf, rows, cols):
    g = pkg.ir.Graph()
    g.sum(g.input("x", [rows, cols]), 0, True)
    (lau,) = cg.lower(g)["launches"]
    assert lau.kind == "sum" and lau.scratch_bytes > 0  # the split path, with runner-allocated scratch
    runner.launch(lau, [x_buf.ptr], out_buf.ptr)
    runner.sync()
    return out_buf.download(cols)


@pytest.mark.parametrize("rows,cols", [(8192, 3000), (4097, 8192)])
def test_static_scratch_colsum_matches_regular_entry_point_twice(pkg, runner, rows, cols):
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    lib = rt.lib()
    rng = np.random.default_rng(rows + cols)
    x_buf = rt.DeviceBuffer(runner, rows * cols * 4)
    a_buf = rt.DeviceBuffer(runner, cols * 4)
    b_buf = rt.DeviceBuffer(runner, cols * 4)
    try:
        for call in range(2):  # the second call runs over the first call's leftover partials
            x = rng.standard_normal(rows * cols).astype(np.float32) * (1 + call)
            x_buf.upload(x)
            want = _regular_colsum(pkg, rt, cg, runner, x_buf, a_buf, rows, cols)
            rt.check(lib.tc_colsum_f32_static(x_buf.ptr, b_buf.ptr, rows, cols, runner.stream()))
            runner.sync()
            got = b_buf.download(cols)
            xs = x.astype(np.float64).reshape(rows, cols)
            gamma = rows * 2.0 ** -24 / (1 - rows * 2.0 ** -24)
            E = gamma * np.abs(xs).sum(axis=0)
            assert np.all(np.abs(got.astype(np.float64) - want) <= 4 * E), f"call {call + 1}"
            assert np.all(np.abs(got.astype(np.float64) - xs.sum(axis=0)) <= 2 * E), f"call {call + 1}"
    finally:
        for b in (x_buf, a_buf, b_buf):
            b.free()


def test_static_scratch_colsum_rejects_oversize(pkg, runner):
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    lib = rt.lib()
    st = lib.tc_colsum_f32_static(256, 256, 2, (1 << 22) + 1, runner.stream())
    assert st == 1
    assert b"above the static scratch maximum" in lib.tc_last_error()
