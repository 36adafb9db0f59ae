"""Tensor parallelism on 2+ GPUs: heads / output groups / wo_b columns / experts /
head rows split over the ranks, partial sums and expert rows exchanged over
NVLink inside the producing and consuming kernels.  Next tokens and every
rank's logits shard must match the single-GPU model.  Runs the self-check
under torchrun; skipped with < 2 GPUs."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


# Every case checks the logits against one GPU by cosine and the served tokens
# against the same tensor-parallel engines stepped directly (next tokens may flip
# against one GPU on near-ties: a different summation order of the split rows).


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("family,moe", [("v4", "ep"), ("v4", "tp"), ("v41", "ep"), ("v41", "tp")])
def test_tp_matches_single_gpu(family, moe):
    """moe="ep": experts owned whole by one rank; moe="tp": every expert split by
    intermediate index over the ranks (partial rows summed in the mHC boundary).
    family "v41": MXFP4 experts, ratio-2/1 compressors and Engram layers."""
    from dsv4_flash_deployment_b200.utils.launch import free_port

    n = 2 if torch.cuda.device_count() < 4 else 4
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           "-m", "dsv4_flash_deployment_b200.parallel.tp_check", "--steps", "3", "--iters", "5", "--moe", moe,
           "--family", family]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=os.path.dirname(os.path.dirname(__file__)))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert '"ok": true' in r.stdout
