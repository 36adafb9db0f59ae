"""CPU tests: scale-chunk layout and the quantization oracle contract."""

import torch

from dsv4_flash_deployment_b200.ops.layout import chunks_to_sf, interleave_w13, sf_to_chunks
from dsv4_flash_deployment_b200.ref import numerics as N


def test_chunk_layout_roundtrip_and_positions():
    sf = torch.randint(0, 255, (300, 20), dtype=torch.int32).to(torch.uint8)
    ch = sf_to_chunks(sf)
    assert ch.shape == (3, 5, 512)
    assert torch.equal(chunks_to_sf(ch, 300, 20), sf)
    # spot-check the byte formula 16*(m%32) + 4*(m//32) + j
    for row, kb in [(0, 0), (37, 6), (130, 19), (255, 3)]:
        rt, m, kt, j = row // 128, row % 128, kb // 4, kb % 4
        assert ch[rt, kt, 16 * (m % 32) + 4 * (m // 32) + j] == sf[row, kb]


def test_act_quant_rules():
    x = torch.tensor([[0.0] * 31 + [448.0 * 3]], dtype=torch.float32)
    q, s = N.act_quant(x)
    assert int(s[0, 0]) == 127 + 2           # 3*448/448 = 3 -> 2^2
    assert float(q[0, -1].float()) == 320.0     # 336 is an e4m3 tie -> even (320)
    tiny = torch.full((1, 32), 1e-9)
    _, s2 = N.act_quant(tiny)                 # amax floor 1e-4 -> 2^ceil(log2(1e-4/448))
    assert int(s2[0, 0]) == 127 + (-22)


def test_fp4_midpoint_ties_to_even():
    s = 1.0
    x = torch.tensor([[0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] + [0.0] * 24]) * s
    codes, scale = N.fp4_act_quant(x, 32, "e8m0")
    # amax 6 -> scale 1; ties go to the even code
    assert codes[0, :8].tolist() == [0, 2, 2, 4, 4, 6, 6, 7]
    assert int(scale[0, 0]) == 127


def test_e2m1_pack_unpack():
    codes = torch.randint(0, 16, (4, 64), dtype=torch.int32).to(torch.uint8)
    assert torch.equal(N.unpack_e2m1(N.pack_e2m1(codes)), codes)


def test_interleave_w13():
    w1 = torch.arange(128 * 2).reshape(128, 2)
    w3 = -torch.arange(128 * 2).reshape(128, 2)
    w = interleave_w13(w1, w3)
    assert torch.equal(w[:64], w1[:64]) and torch.equal(w[64:128], w3[:64])
    assert torch.equal(w[128:192], w1[64:]) and torch.equal(w[192:], w3[64:])


def test_rope_inverse():
    cos, sin = N.rope_table(64, 32, 65536, 160000.0, 16.0, 32, 1)
    x = torch.randn(32, 4, 128)
    y = N.apply_rope(x, cos[:, None], sin[:, None])
    z = N.apply_rope(y, cos[:, None], sin[:, None], inverse=True)
    assert torch.allclose(z, x, atol=1e-5)
    assert torch.equal(y[..., :64], x[..., :64])
