"""The C-ABI library without a GPU: it loads, exports every symbol include/tcb200.h declares,
plans arenas, and NVRTC-compiles generated kernels for sm_100a."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared():
    text = open(os.path.join(ROOT, "include", "tcb200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(tc_[a-z0-9_]+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol(pkg):
    import importlib
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    lib = rt.lib()
    declared = _declared()
    assert len(declared) >= 40
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    # the Python binding types every declared entry point
    assert sorted(set(declared) - set(rt.EXPORTS)) == []
    assert lib.tc_version() == 1


def test_open_without_driver_fails_cleanly(pkg):
    import importlib
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(rt.TcError) as e:
        rt.GpuRunner.create(0)
    assert e.value.status in (2, 7)


def test_arena_planner_never_overlaps_live_buffers(pkg):
    import importlib
    import random
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    r = random.Random(3)
    n = 300
    sizes = [r.randint(1, 1 << 20) for _ in range(n)]
    first = [r.randint(0, 200) for _ in range(n)]
    last = [f + r.randint(0, 40) for f in first]
    offs, total = rt.plan_memory(sizes, first, last)
    assert all(o % 256 == 0 for o in offs)
    for i in range(n):
        assert offs[i] + sizes[i] <= total
        for j in range(i):
            if first[i] <= last[j] and first[j] <= last[i]:
                assert offs[i] + sizes[i] <= offs[j] or offs[j] + sizes[j] <= offs[i]
    # never worse than giving everything its own range
    assert total <= sum((s + 255) // 256 * 256 for s in sizes)


def test_compile_check_reports_errors(pkg):
    import importlib
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    with pytest.raises(rt.TcError) as e:
        rt.compile_check('#include "tcb/common.cuh"\nextern "C" __global__ void k() { this is not cuda; }')
    assert e.value.status == 3


def test_generated_kernels_compile_for_sm100a(pkg):
    """A sample of every template: fused elementwise / rowwise / epilogue, plain gather, reduce rows and columns."""
    import importlib
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    cg = importlib.import_module("tensor-compiler-webgpu_b200.codegen")
    cases = importlib.import_module("tensor-compiler-webgpu_b200.cases").fused_direct_cases()
    pick = [c for c in cases if c["name"] in (
        "a*b+c-d/e [100003]", "x + broadcast(b) [2,4,3,5] <- [2,1,3,1]", "transpose(x) + y [2,3,4] perm [2,0,1]",
        "layernorm [1,4097]", "softmax [2,64]", "log-softmax masked [2,64,64]",
        "matmul naive [2,17,19] x [2,19,33] + bias, gelu")]
    assert len(pick) == 7
    kinds = set()
    for c in pick:
        f = pkg.fuse.fuse(c["graph"])
        for low in (cg.lower_fused(f.graph), cg.lower(c["graph"])):
            for lau in low["launches"]:
                kinds.add(lau.kind)
                assert rt.compile_check(lau.code) > 0
    assert {"fused-elementwise", "fused-rowwise", "fused-epilogue", "gather", "sum", "max", "matmul-naive"} <= kinds
