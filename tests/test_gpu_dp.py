"""Data parallelism on 2 GPUs: torchrun with 2 ranks (NCCL allreduce of the gradients inside libtcb200)
against 1 GPU on the same global batch.  Skipped when fewer than 2 GPUs are visible."""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("buckets", ["4", "1"])
def test_two_ranks_match_one_gpu(tmp_path, buckets):
    """`buckets` 4: the gradient buckets are reduced on the collective stream during the backward; 1: one
    allreduce after it."""
    worker = os.path.join(ROOT, "tests", "dp_worker.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TCB_DP_BUCKETS=buckets)
    one, two = tmp_path / "one.npz", tmp_path / "two.npz"
    subprocess.run([sys.executable, worker, str(one), "2", "8"], check=True, timeout=600, env=env)
    subprocess.run(["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                    "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29517",
                    worker, str(two), "2", "8"], check=True, timeout=700, env=env)
    a, b = np.load(one), np.load(two)
    np.testing.assert_allclose(b["losses"], a["losses"], rtol=1e-5)
    for k in a.files:
        if k != "losses":
            np.testing.assert_allclose(b[k], a[k], rtol=2e-3, atol=2e-5, err_msg=k)
