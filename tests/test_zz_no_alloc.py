"""The allocation-free column sum (tc_colsum_f32_static) against the library's regular reduction.

tc_colsum_f32_static serves callers that cannot allocate device memory where
they need a column sum -- inside a stream capture, under another allocator's
fixed budget, or on a path that cannot take cudaMalloc's device-wide
synchronisation.  Its partial sums live in a static device array, so this test
checks that two calls in a row (the second finding the first call's partials
still in the array) both agree with the regular NVRTC `sum` over axis 0, whose
scratch the runner allocates.  The two use the same per-column order, so for
more than one column they agree bit for bit; a single column is reduced by the
regular path as a row, in another order, and is held to the float32 budget
instead (both within 2E of the exact float64 sum, E = gamma(rows) * sum |x|).

The shapes cover every split the policy takes: one chunk (rows < 64, or at least
75,776 columns), many chunks, and tall narrow matrices whose chunk count is cut
to the grid's 65,535 limit.  This file sorts last so that a run stopping at its
first failure has already run every other test.
"""
import ctypes
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _regular_colsum(pkg, cg, runner, x_buf, out_buf, rows, cols):
    g = pkg.ir.Graph()
    g.sum(g.input("x", [rows, cols]), 0, True)
    (lau,) = cg.lower(g)["launches"]
    assert lau.kind == "sum"
    runner.launch(lau, [x_buf.ptr], out_buf.ptr)
    runner.sync()
    return out_buf.download(cols), lau.info["split"]


@pytest.mark.parametrize("rows,cols,split", [(8192, 3000, 102), (4097, 8192, 37), (63, 5000, 1),
                                             (4, 100000, 1), (300000, 1, 1), (3000000, 2, 65535)])
def test_static_scratch_colsum_matches_regular_entry_point_twice(pkg, runner, rows, cols, split):
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
            want, used = _regular_colsum(pkg, cg, runner, x_buf, a_buf, rows, cols)
            if cols > 1:
                assert used == split
            rt.check(lib.tc_colsum_f32_static(x_buf.ptr, b_buf.ptr, rows, cols, runner.stream()))
            runner.sync()
            got = b_buf.download(cols)
            xs = x.astype(np.float64).reshape(rows, cols)
            gamma = rows * 2.0 ** -24 / (1 - rows * 2.0 ** -24)
            E = gamma * np.abs(xs).sum(axis=0)
            assert np.all(np.abs(got.astype(np.float64) - xs.sum(axis=0)) <= 2 * E), f"call {call + 1}"
            assert np.all(np.abs(want.astype(np.float64) - xs.sum(axis=0)) <= 2 * E), f"call {call + 1}"
            if cols > 1:
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"call {call + 1}"
    finally:
        for b in (x_buf, a_buf, b_buf):
            b.free()


def test_static_scratch_colsum_rejects_oversize(pkg, runner):
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    lib = rt.lib()
    st = lib.tc_colsum_f32_static(256, 256, 2, (1 << 22) + 1, runner.stream())
    assert st == 1
    assert b"above the static scratch maximum" in lib.tc_last_error()


def test_static_scratch_colsum_rejects_host_memory(pkg, runner):
    """Operands must be device memory of the current device: a host pointer is refused on the host,
    before any launch."""
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    lib = rt.lib()
    host = np.zeros(64, np.float32)
    dev = rt.DeviceBuffer(runner, 64 * 4)
    try:
        st = lib.tc_colsum_f32_static(host.ctypes.data, dev.ptr, 8, 8, runner.stream())
        assert st == 1
        assert b"not device memory" in lib.tc_last_error()
    finally:
        dev.free()
