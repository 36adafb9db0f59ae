"""The fused expert-parallel path on one GPU (loopback).

Runs the expert-parallel self-check at world size 1 with the fused transport:
the same dispatch / plan / return-epilogue kernels as on N GPUs, with this GPU
as the only peer, against the model without expert parallelism."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_fused_ep_path_single_gpu_loopback():
    """The fused dispatch / plan / return-epilogue path at world size 1: the same
    kernels (system-scope atomics on the owner's counters, stores into the
    owner's expert rows, W2 rows stored into the source's return buffer, the
    bounded phase waits) with this GPU as the only peer, against the model
    without expert parallelism."""
    from dsv4_flash_deployment_b200.utils.launch import free_port

    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=1", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           "-m", "dsv4_flash_deployment_b200.parallel.ep_check", "--steps", "3", "--iters", "3",
           "--transports", "fused"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=os.path.dirname(os.path.dirname(__file__)))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert '"transport": "fused"' in r.stdout and '"ok": true' in r.stdout
