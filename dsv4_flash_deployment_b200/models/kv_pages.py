"""Paged compressed-KV caches: block pools and block tables, one per compression ratio.

By default every sequence slot owns ``max_seq_len // r`` compressed entries of
every kv-source layer of ratio ``r`` (and as many indexer keys), sized for the
longest request.  In paged mode those caches are pools of blocks of ``block``
entries shared by all slots; slot ``s`` maps compressed entry ``ci`` to pool
row ``table[s][ci // block] * block + ci % block`` (the kernels' ``kv_row``).
All layers of one ratio share one block table, so one reservation covers a
sequence's entries in every layer of that ratio.  The reference serves behind
vLLM's paged KV manager (``--block-size``, ``--gpu-memory-utilization``;
``kernel-optimizations-recipe/dsv41-flash-v6e16-serving.yaml:360-373``); this
applies the same idea to the compressed caches (the sliding-window ring stays
per slot: it is ``sliding_window`` rows whatever the length).

Admission reserves every block a request can touch (prompt + new tokens, one
group of margin) for each ratio, or none; a running sequence therefore never
runs out of blocks and nothing is preempted.  Finishing returns them.
Unmapped table entries (free slots, the padding slot) point at one scratch
block past the allocator's range, so padding rows stay inside the pool.

The free list and the host table live in the native allocator
(``csrc/host/kv_blocks.cpp``); this class mirrors the tables to the device
when they change (before the next step's launches, on the step stream).
"""

from __future__ import annotations

import numpy as np
import torch

from ..ops.host import KvBlockAllocator


class KvPager:
    def __init__(self, cfg, dev, n_slots: int, max_seq_len: int, block: int, pool_tokens: int = 0):
        if block <= 0 or block & (block - 1):
            raise ValueError(f"kv block size must be a power of two, got {block}")
        self.block = block
        self.shift = block.bit_length() - 1
        self.n_slots = n_slots                       # including the padding slot
        self.max_seq_len = max_seq_len
        self.pool_tokens = pool_tokens or (n_slots - 1) * max_seq_len
        self.ratios = sorted({cfg.ratio(l) for l in cfg.kv_source_layer_ids})
        self.alloc: dict[int, KvBlockAllocator] = {}
        self.host: dict[int, np.ndarray] = {}
        self.table: dict[int, torch.Tensor] = {}
        self.desc: dict[int, torch.Tensor] = {}
        self.max_c: dict[int, int] = {}
        self.n_blocks: dict[int, int] = {}
        for r in self.ratios:
            max_c = max(1, max_seq_len // r)
            ld = -(-max_c // block)
            nb = max(1, -(-max(1, self.pool_tokens // r) // block))
            self.alloc[r] = KvBlockAllocator(nb, n_slots, ld)
            self.host[r] = np.full((n_slots, ld), nb, np.int32)          # nb = the scratch block
            self.table[r] = torch.from_numpy(self.host[r].copy()).to(dev)
            self.desc[r] = torch.tensor([self.table[r].data_ptr(), ld, self.shift, max_c], dtype=torch.int64)
            self.max_c[r] = max_c
            self.n_blocks[r] = nb
        self._dirty: set[int] = set()

    # pool geometry
    def rows(self, r: int) -> int:
        """Physical rows of a ratio-``r`` pool (the allocator's blocks + the scratch block)."""
        return (self.n_blocks[r] + 1) * self.block

    def blocks_for(self, r: int, total_len: int) -> int:
        entries = min(self.max_c[r], total_len // r + 1)
        return -(-entries // self.block)

    # admission
    def fits(self, total_len: int) -> bool:
        """Whether a request of ``total_len`` tokens can ever be admitted (empty pools)."""
        return all(self.blocks_for(r, total_len) <= self.n_blocks[r] for r in self.ratios)

    def reserve(self, slot: int, total_len: int) -> bool:
        need = {r: self.blocks_for(r, total_len) for r in self.ratios}
        if any(self.alloc[r].free_blocks < n - self.alloc[r].slot_blocks(slot) for r, n in need.items()):
            return False
        for r, n in need.items():
            if not self.alloc[r].reserve(slot, n):
                raise RuntimeError("block allocator refused a checked reservation")
            row = self.alloc[r].row(slot)
            self.host[r][slot] = np.where(row >= 0, row, self.n_blocks[r])
            self._dirty.add(r)
        return True

    def release(self, slot: int) -> None:
        for r in self.ratios:
            self.alloc[r].release(slot)
            self.host[r][slot] = self.n_blocks[r]
            self._dirty.add(r)

    def free_blocks(self) -> dict[int, int]:
        return {r: self.alloc[r].free_blocks for r in self.ratios}

    def sync(self) -> None:
        """Copies changed tables to the device on the current stream (ordered before the step)."""
        for r in sorted(self._dirty):
            self.table[r].copy_(torch.from_numpy(self.host[r]))
        self._dirty.clear()
