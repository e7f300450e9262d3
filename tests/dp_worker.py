"""One rank of the data-parallel check (launched by tests/test_gpu_dp.py through torch.distributed.run).

Each rank trains the small C5-shaped model on its shard of a fixed global
batch for `steps` steps through DPTrainer (gradients allreduced over NCCL by
libtcb200), then rank 0 writes the losses and final parameters to `out`.
"""
import importlib
import os
import sys
from datetime import timedelta

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(out, steps, batch):
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    pkg = importlib.import_module("tensor-compiler-webgpu_b200")
    rt = importlib.import_module("tensor-compiler-webgpu_b200.runtime")
    wl = importlib.import_module("tensor-compiler-webgpu_b200.workloads")
    dp = importlib.import_module("tensor-compiler-webgpu_b200.dp")
    cfg, c = wl.c5_cfg(d=64, L=2, H=4, ff=128, T=32, batch=batch)
    V = c["V"]
    bl = batch // world
    runner = rt.GpuRunner.create(local)
    comm = dp.Comm(runner, rank, world) if world > 1 else None
    params = pkg.steps.init_params_normal(V, 0, 0.02, cfg)
    tr = dp.DPTrainer(runner, V, bl, cfg, params, comm=comm)
    toks = wl.c5_tokens(batch, cfg["T"], V)[rank * bl:(rank + 1) * bl]
    x, y = wl.one_hot_batch(toks, V)
    losses = [tr.train(x, y) for _ in range(steps)]
    if world > 1:
        import torch
        t = torch.tensor(losses, dtype=torch.float64)
        dist.all_reduce(t)
        losses = list((t / world).numpy())
    if rank == 0:
        p = tr.read(tr.names)
        np.savez(out, losses=np.array(losses), **{k.replace(".", "_"): v for k, v in p.items()})
    tr.destroy()
    if comm:
        comm.destroy()
    runner.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], int(sys.argv[2]), int(sys.argv[3]))
