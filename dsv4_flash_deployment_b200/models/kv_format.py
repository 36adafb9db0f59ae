"""Byte layouts of the attention caches.

Every cached attention row has already been through a quantize-dequantize
round trip in the reference; the caches store the quantized form itself:

* KV8 -- sliding-window rows (and this step's rows): ``head_dim`` e4m3 codes,
  then one ue8m0 scale byte per 32 columns.  This is the FP8 / ue8m0-per-32
  round trip of the window KV (``tpu-v7x/deepseek_v41/reference.py:741``,
  ``act_quant(kv, 32, ue8m0)``): 528 bytes per 512-dim row instead of 1,024.
* IK4 -- indexer keys: ``head_dim / 2`` bytes of e2m1 codes (same packing),
  then one ue8m0 scale byte per 32 columns: the e2m1 / ue8m0-per-32 round trip
  of the indexer key (``reference.py:638``): 68 bytes per 128-dim key instead
  of 256.  The indexer reads every key of the context, so this is the read
  that grows with context length.
* KV4 -- compressed rows: ``head_dim / 2`` bytes of e2m1 codes (column 2i in
  the low nibble of byte i, column 2i+1 in the high nibble, the checkpoint's
  packing), then one e4m3 scale byte per 16 columns.  This is the e2m1 /
  e4m3-per-16 round trip of the compressed latent (``reference.py:801``):
  288 bytes per row instead of 1,024.

All three decode to exactly the values a bf16 cache held: an e4m3 code or an
e2m1 code times a power of two, and an e2m1 code times an e4m3 scale, have at
most 6 significant bits,
which bf16's 8-bit significand represents exactly.  The TPU serving patches
store a comparable FP8 record (448 e4m3 + 7 ue8m0 + 64 bf16 RoPE dims,
``kernel-optimizations-recipe/patches/tpu-inference/0003-*.patch:330-342``);
this layout keeps the reference model's own rounding of every column instead.
"""

from __future__ import annotations

import torch

from ..ref import numerics as N


def kv8_bytes(head_dim: int) -> int:
    return head_dim + head_dim // 32


def kv4_bytes(head_dim: int) -> int:
    return head_dim // 2 + head_dim // 16


def ik4_bytes(head_dim: int) -> int:
    return head_dim // 2 + head_dim // 32


def kv4_dim(row_bytes: int) -> int:
    """Head dim of a KV4 row of ``row_bytes`` bytes."""
    if (row_bytes * 16) % 9:
        raise ValueError(f"{row_bytes} is not a KV4 row width")
    return row_bytes * 16 // 9


def kv8_encode(x: torch.Tensor) -> torch.Tensor:
    """[..., d] values -> [..., kv8_bytes(d)] uint8 records (quantizes like ``act_quant``)."""
    q, s = N.act_quant(x, 32)
    return torch.cat([q.view(torch.uint8), s.to(torch.uint8)], -1)


def kv8_decode(rec: torch.Tensor, head_dim: int) -> torch.Tensor:
    """[..., kv8_bytes(d)] uint8 -> [..., d] fp32."""
    q = rec[..., :head_dim].contiguous().view(torch.float8_e4m3fn)
    s = rec[..., head_dim:head_dim + head_dim // 32]
    return N.act_dequant(q, s, 32)


def kv4_encode(x: torch.Tensor) -> torch.Tensor:
    """[..., d] values -> [..., kv4_bytes(d)] uint8 records (e2m1 codes, e4m3 scale per 16)."""
    codes, s = N.fp4_act_quant(x, 16, "e4m3")
    return torch.cat([N.pack_e2m1(codes), s.view(torch.uint8)], -1)


def kv4_decode(rec: torch.Tensor, head_dim: int) -> torch.Tensor:
    """[..., kv4_bytes(d)] uint8 -> [..., d] fp32."""
    codes = N.unpack_e2m1(rec[..., :head_dim // 2])
    s = rec[..., head_dim // 2:head_dim // 2 + head_dim // 16].contiguous().view(torch.float8_e4m3fn)
    return N.fp4_dequant(codes, s, 16)


def ik4_encode(x: torch.Tensor) -> torch.Tensor:
    """[..., d] values -> [..., ik4_bytes(d)] uint8 records (e2m1 codes, ue8m0 scale per 32)."""
    codes, s = N.fp4_act_quant(x, 32, "e8m0")
    return torch.cat([N.pack_e2m1(codes), s.to(torch.uint8)], -1)


def ik4_decode(rec: torch.Tensor, head_dim: int) -> torch.Tensor:
    """[..., ik4_bytes(d)] uint8 -> [..., d] fp32."""
    codes = N.unpack_e2m1(rec[..., :head_dim // 2])
    s = rec[..., head_dim // 2:head_dim // 2 + head_dim // 32].contiguous()
    return N.fp4_dequant(codes, s, 32)
