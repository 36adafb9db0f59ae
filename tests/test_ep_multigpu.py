"""Expert parallelism on 2+ GPUs: every transport (NCCL all-to-all baseline,
NVLink peer stores with bounded signal waits, and the fused dispatch that
stores straight into the owners' expert rows and returns rows from the W2
epilogue) must reproduce the single-GPU model's logits.  Runs the self-check under torchrun; skipped with < 2 GPUs."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_transports_match_single_gpu():
    from dsv4_flash_deployment_b200.utils.launch import free_port

    n = min(torch.cuda.device_count(), 4)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           "-m", "dsv4_flash_deployment_b200.parallel.ep_check", "--steps", "3", "--iters", "5"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=os.path.dirname(os.path.dirname(__file__)))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert '"transport": "p2p"' in r.stdout and '"transport": "fused"' in r.stdout
    assert '"ok": false' not in r.stdout and r.stdout.count('"ok": true') == 3


