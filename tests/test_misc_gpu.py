"""Small device kernels vs plain PyTorch references: row argmax (single- and multi-CTA rows)."""

import pytest
import torch

from dsv4_flash_deployment_b200.ops import _ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 3, 40, 200])
@pytest.mark.parametrize("V", [1000, 129280, 129283])
def test_argmax_rows_matches_torch(T, V):
    ext = _ext.load()
    torch.manual_seed(T * 7 + V)
    ld = (V + 127) // 128 * 128 + (1 if V % 2 else 0)   # odd V: unaligned rows take the scalar path
    logits = torch.randn(T, ld, device="cuda")
    # ties: the first index wins
    logits[:, 5] = 9.0
    logits[:, V - 3] = 9.0
    logits[T // 2, :] = 0.0
    logits[T // 2, V - 1] = 1.0
    scratch = torch.zeros(2 * max(T, 296) + 256, dtype=torch.int32, device="cuda")
    for use_scratch in (False, True):
        out = torch.full((T,), -1, dtype=torch.int32, device="cuda")
        for _ in range(3):   # counters must come back to zero between calls
            ext.argmax_rows(logits, T, V, out, scratch if use_scratch else None, None, 0)
        want = torch.argmax(logits[:, :V], dim=1).int()
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    assert int(scratch[-256:].abs().sum()) == 0
