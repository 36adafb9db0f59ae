"""Quantized cache records (CPU): KV8 / KV4 rows decode to exactly the values of the
reference's round trips (FP8 / ue8m0 per 32 for window rows, e2m1 / e4m3 per 16 for
compressed rows), and those values are exact in bf16, so a record cache serves the
same attention inputs as a bf16 cache of round-tripped rows."""

import torch

from dsv4_flash_deployment_b200.models.kv_format import (kv4_bytes, kv4_decode, kv4_dim, kv4_encode, kv8_bytes,
                                                         kv8_decode, kv8_encode)
from dsv4_flash_deployment_b200.ref import numerics as N


def _rows(n=64, d=512, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, d, generator=g) * torch.logspace(-3, 2, n)[:, None]
    x[3, :40] = 0.0                      # an all-zero scale block
    x[5, 7] = 1e3                        # an outlier in one block (e4m3 scale range: amax <= 6 * 448)
    return x.to(torch.bfloat16)


def test_sizes():
    assert kv8_bytes(512) == 528 and kv4_bytes(512) == 288
    assert kv8_bytes(512) % 16 == 0 and kv4_bytes(512) % 16 == 0
    assert kv4_dim(288) == 512


def test_kv8_record_is_the_fp8_round_trip():
    x = _rows()
    rec = kv8_encode(x)
    assert rec.dtype == torch.uint8 and rec.shape == (64, 528)
    dec = kv8_decode(rec, 512)
    want = N.act_quant_roundtrip(x)
    assert torch.equal(dec.to(torch.bfloat16), want)
    assert torch.equal(dec, dec.to(torch.bfloat16).float())     # exact in bf16


def test_kv8_reencoding_a_round_tripped_row_keeps_its_values():
    # ring rows are copied as records; a writer that re-quantizes the decoded row
    # (e.g. a rebuilt cache) must land on the same values
    x = N.act_quant_roundtrip(_rows(seed=1))
    assert torch.equal(kv8_decode(kv8_encode(x), 512).to(torch.bfloat16), x)


def test_kv4_record_is_the_fp4_round_trip():
    x = _rows(seed=2)
    rec = kv4_encode(x)
    assert rec.shape == (64, 288)
    dec = kv4_decode(rec, 512)
    want = N.fp4_act_quant_roundtrip(x, 16, "e4m3")
    assert torch.equal(dec.to(torch.bfloat16), want)
    assert torch.equal(dec, dec.to(torch.bfloat16).float())


def test_kv4_nibble_order_is_the_checkpoint_packing():
    x = torch.zeros(1, 512)
    x[0, 0], x[0, 1] = 6.0, -0.5          # codes 7 and 0b1001 at scale 1
    x[0, 2:16] = 1.0
    rec = kv4_encode(x.to(torch.bfloat16))
    assert int(rec[0, 0]) == (7 | (9 << 4))
    assert torch.equal(rec[0, 256:257].view(torch.float8_e4m3fn).float(), torch.tensor([1.0]))


def test_record_caches_are_smaller():
    d = 512
    assert kv8_bytes(d) / (2 * d) < 0.52 and kv4_bytes(d) / (2 * d) < 0.29


def test_ik4_record_is_the_indexer_key_round_trip():
    from dsv4_flash_deployment_b200.models.kv_format import ik4_bytes, ik4_decode, ik4_encode

    x = _rows(d=128, seed=3)
    rec = ik4_encode(x)
    assert ik4_bytes(128) == 68 and rec.shape == (64, 68)
    dec = ik4_decode(rec, 128)
    assert torch.equal(dec.to(torch.bfloat16), N.fp4_act_quant_roundtrip(x, 32, "e8m0"))
    assert torch.equal(dec, dec.to(torch.bfloat16).float())
