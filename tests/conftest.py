"""Shared fixtures: the package (imported by its directory name), the oracle, the GPU marker."""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
ORACLE_DIR = os.path.join(ROOT, "oracle")
if ORACLE_DIR not in sys.path:
    sys.path.insert(0, ORACLE_DIR)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the C-ABI library on cuda:0)")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module("tensor-compiler-webgpu_b200")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o  # noqa: the checker, never the thing measured
    o.build()
    return o


@pytest.fixture(scope="session")
def runner(pkg):
    """One GPU context for the session.  On a machine without a B200 this errors: there is no CPU fallback."""
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    r = rt.GpuRunner.create(0)
    yield r
    r.close()
