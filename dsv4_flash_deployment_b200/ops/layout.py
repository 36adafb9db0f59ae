"""Host-side layout transforms for block-scaled operands (pure torch, any device).

The GEMM kernels read ue8m0 block scales in a 512-byte "chunk" layout: one
chunk per (128-row tile, 128-column k tile); inside a chunk, row ``m`` of the
tile and k-block ``j`` (32 columns) sit at byte ``16*(m%32) + 4*(m//32) + j``.
That is the shared-memory image the tensor core's ``tcgen05.cp 32x128b.warpx4``
copy turns into the TMEM scale-factor layout of a 128-row MMA.
"""

from __future__ import annotations

import torch


def ceil_to(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def expand_block_scales(scale: torch.Tensor, rows: int, block: int = 32) -> torch.Tensor:
    """[rows/32, K/32] (32x32-block) or [rows, K/32] (per-row) -> per-row [rows, K/32]."""
    if scale.shape[0] == rows:
        return scale
    return scale.repeat_interleave(block, 0)[:rows]


def sf_to_chunks(sf_rows: torch.Tensor, rows_pad: int | None = None) -> torch.Tensor:
    """Per-row scales [R, K/32] (uint8) -> chunk layout [R_pad/128, K_pad/128, 512]."""
    r, kb = sf_rows.shape
    rp = ceil_to(rows_pad or r, 128)
    kbp = ceil_to(kb, 4)
    full = torch.full((rp, kbp), 127, dtype=torch.uint8, device=sf_rows.device)
    full[:r, :kb] = sf_rows
    # (rt, g=m//32, i=m%32, kt, j) -> (rt, kt, i, g, j)
    c = full.reshape(rp // 128, 4, 32, kbp // 4, 4).permute(0, 3, 2, 1, 4).contiguous()
    return c.reshape(rp // 128, kbp // 4, 512)


def chunks_to_sf(chunks: torch.Tensor, rows: int, kblocks: int) -> torch.Tensor:
    """Inverse of :func:`sf_to_chunks` (for tests)."""
    rt, kt, _ = chunks.shape
    c = chunks.reshape(rt, kt, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(rt * 128, kt * 4)
    return c[:rows, :kblocks]


def interleave_w13(w1: torch.Tensor, w3: torch.Tensor, block: int = 64) -> torch.Tensor:
    """[I, K] gate + [I, K] up -> [2I, K] with 128-row tiles = [64 gate; 64 up] rows."""
    i = w1.shape[0]
    assert i % block == 0
    a = w1.reshape(i // block, block, *w1.shape[1:])
    b = w3.reshape(i // block, block, *w3.shape[1:])
    return torch.cat([a, b], 1).reshape(2 * i, *w1.shape[1:])
