"""The differential fuzzer on a fixed 20% sample of the corpus (programs i with i % 10 in {1, 2}):
every run's fused and unfused GPU results within amendment 8's budget of the float64 oracle
(the reference recorded 5318/5318 over the whole corpus; tests/fuzz_m4.py runs all of it)."""
import importlib

import pytest

import fuzz_m4

pytestmark = pytest.mark.gpu


def test_fuzz_sample(pkg, runner):
    co = importlib.import_module("tensor-compiler-webgpu_b200.corpus")
    progs = fuzz_m4.select(10)
    fuzz_m4.precompile(pkg, co, progs)
    res = fuzz_m4.run_fuzz(runner, progs)
    assert res["runs"] > 900
    assert res["failures"] == [], res["failures"][:3]
    assert res["fusedPassed"] == res["runs"] and res["unfusedPassed"] == res["runs"]
