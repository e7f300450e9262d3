"""The library's NCCL bootstrap gives up with an error when a peer never joins (no GPU work involved).

tc_comm_init builds a non-blocking communicator and waits for it with a bound: with world size 2 and
no second rank, the wait must run out and return TC_ERR_TIMEOUT (after aborting the half-built
communicator), well within the caller's limit, instead of hanging the process.  Only host-side
bootstrap runs -- no kernel or collective is launched -- and it runs in a child process with its own
time limit so a stuck abort could not stall the test session.
"""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CHILD = r"""
import ctypes, importlib, json, sys, time
sys.path.insert(0, sys.argv[1])
rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
lib = rt.lib()
runner = rt.GpuRunner.create(0)
uid = ctypes.create_string_buffer(128)
st = lib.tc_comm_unique_id(uid)
h = ctypes.c_void_p()
t0 = time.monotonic()
rc = lib.tc_comm_init(runner.ctx, 0, 2, uid, 2000, ctypes.byref(h)) if st == 0 else -1
dt = time.monotonic() - t0
print(json.dumps({"unique_id": st, "rc": rc, "seconds": dt, "msg": lib.tc_last_error().decode(errors="replace")}))
runner.close()
"""


def test_comm_init_without_a_peer_times_out():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    p = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, timeout=120, env=env)
    assert p.returncode == 0, p.stderr[-2000:]
    out = json.loads(p.stdout.strip().splitlines()[-1])
    assert out["unique_id"] == 0, out
    assert out["rc"] == 5, out          # TC_ERR_TIMEOUT
    assert "not complete after 2000 ms" in out["msg"], out
    assert out["seconds"] < 30, out
