"""Tensor-parallel weight slicing on the host (CPU only): the expert split's
W13 row blocks keep each (gate, up) pair of 64 intermediate indices together and
its W2 column slices line up with them; scale chunks follow their rows and
columns; head-row shards cover the padded vocabulary."""

import pytest
import torch

from dsv4_flash_deployment_b200.models.weights import ExpertBlock
from dsv4_flash_deployment_b200.ops.gemm import MxWeight, prepare_w13
from dsv4_flash_deployment_b200.ops.layout import chunks_to_sf
from dsv4_flash_deployment_b200.parallel.tp import TPGroup, mx_cols, mx_rows


def _block(E=3, I=512, D=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = lambda n, k: (torch.randn(n, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
    s = lambda n, k: torch.randint(118, 123, (n, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
    w1 = [(w(I, D), s(I, D)) for _ in range(E)]
    w3 = [(w(I, D), s(I, D)) for _ in range(E)]
    w2 = [(w(D, I), s(D, I)) for _ in range(E)]
    m13 = [prepare_w13(a[0], a[1], b[0], b[1], "cpu") for a, b in zip(w1, w3)]
    w13 = MxWeight(torch.cat([m.q for m in m13]), torch.cat([m.sf for m in m13]), E * 2 * I, D, m13[0].kind)
    m2 = [MxWeight.from_checkpoint(a, b, "cpu") for a, b in w2]
    w2m = MxWeight(torch.cat([m.q for m in m2]), torch.cat([m.sf for m in m2]), E * D, I, m2[0].kind)
    return ExpertBlock(w13, w2m, E, I), w1, w3, w2


@pytest.mark.parametrize("world", [2, 4])
def test_expert_split_slices_match_the_whole_expert(world):
    E, I, D = 3, 512, 256
    ex, w1, w3, w2 = _block(E, I, D)
    il = I // world
    for r in range(world):
        part = TPGroup(r, world, None, "cpu", moe="tp").shard_experts(ex)
        assert part.inter == il and part.w13.n == E * 2 * il and part.w2.k == il
        q13 = part.w13.q.view(torch.uint8)
        for e in range(E):
            rows = q13[e * 2 * il:(e + 1) * 2 * il]
            # 128-row blocks = [64 gate rows; 64 up rows] of intermediate indices r*il + 64b ...
            for b in range(2 * il // 128):
                i0 = r * il + 64 * b
                assert torch.equal(rows[128 * b:128 * b + 64], w1[e][0][i0:i0 + 64].view(torch.uint8))
                assert torch.equal(rows[128 * b + 64:128 * b + 128], w3[e][0][i0:i0 + 64].view(torch.uint8))
            cols = part.w2.q.view(torch.uint8)[e * D:(e + 1) * D]
            assert torch.equal(cols, w2[e][0][:, r * il:(r + 1) * il].view(torch.uint8))
        sf2 = chunks_to_sf(part.w2.sf, E * D, il // 32)
        full2 = chunks_to_sf(ex.w2.sf, E * D, I // 32)
        assert torch.equal(sf2, full2[:, r * il // 32:(r + 1) * il // 32])


def test_row_and_column_slices_and_head_rows():
    ex, *_ = _block()
    w = ex.w2
    top = mx_rows(w, 128, 384)
    assert top.n == 256 and torch.equal(top.q, w.q[128:384]) and torch.equal(top.sf, w.sf[1:3])
    left = mx_cols(w, 256, 512)
    assert left.k == 256 and torch.equal(left.q.view(torch.uint8), w.q[:, 256:512].view(torch.uint8))
    with pytest.raises(AssertionError):
        mx_cols(w, 64, 192)
    vocab = 1000
    shards = [TPGroup(r, 4, None, "cpu").vocab_rows(vocab) for r in range(4)]
    assert all(rows % 128 == 0 for _, rows in shards)
    assert shards[0][0] == 0 and sum(rows for _, rows in shards) >= vocab
    assert all(shards[i][0] + shards[i][1] == shards[i + 1][0] for i in range(3))
