"""The data-parallel path's host logic with world size 2 on CPU (gloo), no GPU.

* Sharding the batch and averaging the per-rank gradients (allreduce sum x 1/W)
  gives the full-batch gradient: each rank evaluates its shard's gradient graph
  on the float64 oracle, the ranks allreduce over gloo, and the result matches
  the oracle's full-batch gradient.
* The NCCL unique id reaches every rank through the gloo bootstrap.
* A rank that never joins makes the others fail with an error, not hang.
"""
import importlib
import os
import socket
import sys

import numpy as np
import pytest

from conftest import ROOT

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, world, port, timeout_s=60):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))


def _shard_worker(rank, world, port, q):
    _setup(rank, world, port)
    import oracle
    pkg = importlib.import_module("tensor-compiler-webgpu_b200")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=16, L=1, H=2, ff=32, T=8, batch=4)
    V, B = c["V"], c["batch"]
    bl = B // world
    params = s.init_params_normal(V, 0, 0.02, cfg)
    toks = wl.c5_tokens(B, cfg["T"], V)[rank * bl:(rank + 1) * bl]
    x, y = wl.one_hot_batch(toks, V)
    gs = s.build_grad3b(V, bl, cfg)
    vals = oracle.evaluate(gs["graph"], {**params, "x": x, "y": y, gs["cotangent"]: [1.0]})
    flat = np.concatenate([vals[gs["grads"][n]] for n in gs["names"]])
    t = torch.from_numpy(flat.copy())
    dist.all_reduce(t)
    t /= world
    if rank == 0:
        q.put(t.numpy())
    dist.destroy_process_group()


def test_sharded_gradients_average_to_the_full_batch_gradient(oracle, pkg):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    mp.start_processes(_shard_worker, args=(world, port, q), nprocs=world, start_method="spawn", join=True)
    got = q.get(timeout=10)
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=16, L=1, H=2, ff=32, T=8, batch=4)
    V, B = c["V"], c["batch"]
    params = s.init_params_normal(V, 0, 0.02, cfg)
    x, y = wl.one_hot_batch(wl.c5_tokens(B, cfg["T"], V), V)
    gs = s.build_grad3b(V, B, cfg)
    vals = oracle.evaluate(gs["graph"], {**params, "x": x, "y": y, gs["cotangent"]: [1.0]})
    want = np.concatenate([vals[gs["grads"][n]] for n in gs["names"]])
    np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-14)


def _uid_worker(rank, world, port, q):
    _setup(rank, world, port)
    box = [os.urandom(128) if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    q.put((rank, box[0]))
    dist.destroy_process_group()


def test_unique_id_bootstrap_reaches_every_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_uid_worker, args=(world, _port(), q), nprocs=world, start_method="spawn", join=True)
    got = dict(q.get(timeout=10) for _ in range(world))
    assert len(got[0]) == 128 and got[0] == got[1]


def _lonely_worker(rank, world, port, q):
    try:
        _setup(rank, world, port, timeout_s=3)
        q.put("joined")
    except Exception as exc:  # the missing peer surfaces as an error on the host
        q.put(type(exc).__name__)


def test_a_rank_that_never_joins_fails_the_others_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_worker, args=(0, 2, _port(), q))
    p.start()
    p.join(60)
    assert not p.is_alive()
    assert q.get(timeout=5) != "joined"


def _prescaled_worker(rank, world, port, q):
    """The product's algebra for a power-of-two world (dp.py): each rank seeds its loss cotangent with 1/W
    instead of 1, and the allreduce is a plain sum with no division afterwards."""
    _setup(rank, world, port)
    import oracle
    pkg = importlib.import_module("tensor-compiler-webgpu_b200")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=16, L=1, H=2, ff=32, T=8, batch=4)
    V, B = c["V"], c["batch"]
    bl = B // world
    params = s.init_params_normal(V, 0, 0.02, cfg)
    toks = wl.c5_tokens(B, cfg["T"], V)[rank * bl:(rank + 1) * bl]
    x, y = wl.one_hot_batch(toks, V)
    gs = s.build_grad3b(V, bl, cfg)
    feed = {**params, "x": x, "y": y}
    seeded = oracle.evaluate(gs["graph"], {**feed, gs["cotangent"]: [1.0 / world]})
    plain = oracle.evaluate(gs["graph"], {**feed, gs["cotangent"]: [1.0]})
    mine = np.concatenate([seeded[gs["grads"][n]] for n in gs["names"]])
    unit = np.concatenate([plain[gs["grads"][n]] for n in gs["names"]])
    t = torch.from_numpy(mine.copy())
    dist.all_reduce(t)  # a plain sum: the 1/W is already inside every rank's gradients
    if rank == 0:  # small messages only: the parent reads the queue after the ranks have exited
        q.put((t.numpy(), bool(np.array_equal(mine, unit / world))))
    dist.destroy_process_group()


def test_prescaled_seed_plain_sum_gives_the_full_batch_gradient(oracle, pkg):
    """Backpropagation is linear in the cotangent seed and a power-of-two scale is exact in every
    floating-point operation (away from underflow), so seeding with 1/W gives exactly 1/W times the
    unit-seed gradients, bit for bit; their plain sum over the ranks is the full-batch gradient."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_prescaled_worker, args=(world, _port(), q), nprocs=world, start_method="spawn", join=True)
    got, exact = q.get(timeout=10)
    assert exact
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    s = pkg.steps
    cfg, c = wl.c5_cfg(d=16, L=1, H=2, ff=32, T=8, batch=4)
    V, B = c["V"], c["batch"]
    params = s.init_params_normal(V, 0, 0.02, cfg)
    x, y = wl.one_hot_batch(wl.c5_tokens(B, cfg["T"], V), V)
    gs = s.build_grad3b(V, B, cfg)
    vals = oracle.evaluate(gs["graph"], {**params, "x": x, "y": y, gs["cotangent"]: [1.0]})
    want = np.concatenate([vals[gs["grads"][n]] for n in gs["names"]])
    np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-14)
