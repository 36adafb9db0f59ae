"""Failure detection on the GPU without a fault: every spin on a peer's signal is
bounded (2 s of %globaltimer); when it runs out the kernel records
ERR_PEER_TIMEOUT in the device error word and returns, the host raises, and the
context stays usable.  The "peers" here are local buffers that nothing ever
signals (one GPU, no other rank involved)."""

import time

import pytest
import torch

from dsv4_flash_deployment_b200.ops import _ext
from dsv4_flash_deployment_b200.ops.gemm import ErrorWord

pytestmark = pytest.mark.gpu

ERR_PEER_TIMEOUT, KID_COMM = 2, 4


def _expect_timeout(run):
    dev = "cuda"
    ErrorWord.get(dev).zero_()
    t0 = time.time()
    run()
    torch.cuda.synchronize()
    dt = time.time() - t0
    with pytest.raises(RuntimeError) as ei:
        ErrorWord.check(dev)
    msg = str(ei.value)
    assert f"code={ERR_PEER_TIMEOUT}" in msg and f"kernel={KID_COMM}" in msg, msg
    assert 1.5 < dt < 30, dt
    # the context is still healthy: a kernel after the timeout runs and is correct
    x = torch.randn(4, 300, device=dev)
    out = torch.empty(4, dtype=torch.int32, device=dev)
    _ext.load().argmax_rows(x, 4, 300, out, None, None, 0)
    torch.cuda.synchronize()
    assert torch.equal(out, x.argmax(1).int())
    ErrorWord.check(dev)


def test_expert_exchange_wait_times_out_and_reports():
    """ep_wait on signal words no peer ever writes (epoch 1 > 0)."""
    ext = _ext.load()
    world = 2
    sig = torch.zeros(2 * world, dtype=torch.int32, device="cuda")
    epoch = torch.ones(2, dtype=torch.int32, device="cuda")
    _expect_timeout(lambda: ext.ep_wait(sig, world, 0, epoch, ErrorWord.get("cuda")))


def test_tensor_parallel_merge_wait_times_out_and_reports():
    """tp_argmax_merge publishes its own pairs, then waits for a second "rank"
    whose signal slot nothing sets."""
    ext = _ext.load()
    world, S = 2, 3
    sig_a = torch.zeros(3 * world, dtype=torch.int32, device="cuda")      # this rank's signal array
    sig_b = torch.zeros(3 * world, dtype=torch.int32, device="cuda")      # the silent peer's
    done = torch.zeros(3, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(3, dtype=torch.int32, device="cuda")
    peer_sig = torch.tensor([sig_a.data_ptr(), sig_b.data_ptr()], dtype=torch.int64, device="cuda")
    vals = torch.zeros(S, device="cuda")
    idx = torch.zeros(S, dtype=torch.int32, device="cuda")
    peer_val = torch.tensor([vals.data_ptr(), vals.data_ptr()], dtype=torch.int64, device="cuda")
    peer_idx = torch.tensor([idx.data_ptr(), idx.data_ptr()], dtype=torch.int64, device="cuda")
    phase = 2
    sync = torch.tensor([peer_sig.data_ptr(), sig_a.data_ptr(), done.data_ptr() + 4 * phase,
                         epoch.data_ptr() + 4 * phase, phase, world, 0], dtype=torch.int64)
    out = torch.full((S,), -1, dtype=torch.int32, device="cuda")
    _expect_timeout(lambda: ext.tp_argmax_merge(sync, peer_val, peer_idx, S, out, ErrorWord.get("cuda")))
    # its own publish did land: slot (phase, rank 0) of both signal arrays holds epoch 1
    assert int(sig_a[phase * world]) == 1 and int(sig_b[phase * world]) == 1
