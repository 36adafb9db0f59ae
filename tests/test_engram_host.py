"""Native Engram hashing and host row gather vs the numpy oracle."""

import numpy as np
import torch

from dsv4_flash_deployment_b200.config import v41_flash_config, v41_tiny_config
from dsv4_flash_deployment_b200.ops import host
from dsv4_flash_deployment_b200.ref.engram import EngramHasher


def _check(cfg, n_tok, seed, dead_frac=0.0):
    h = EngramHasher(cfg)
    rng = np.random.default_rng(seed)
    hist = h.compress(rng.integers(0, cfg.vocab_size, n_tok))
    if dead_frac:
        hist = np.where(rng.random(n_tok) < dead_frac, -1, hist)
    pos = rng.permutation(n_tok)[: max(1, n_tok // 2)]
    want = h.hash(hist, pos)
    got = host.engram_hash(hist, pos, h.mult, h.layout.primes, h.layout.offsets, h.pad, threads=4)
    assert got.shape == want.shape and np.array_equal(got, want)


def test_hash_tiny_config():
    _check(v41_tiny_config(), 300, 0)
    _check(v41_tiny_config(), 64, 1, dead_frac=0.1)


def test_hash_full_v41_layout():
    # full V4.1 tables: 16M-vocab primes, int64 products that wrap
    _check(v41_flash_config(), 2000, 2)


def test_gather_rows_masks_out_of_range():
    t = torch.randint(0, 255, (50, 264), dtype=torch.uint8)
    ids = np.array([3, -1, 49, 50, 7])
    out = host.gather_rows(t, ids, threads=2)
    assert torch.equal(out[0], t[3]) and torch.equal(out[2], t[49]) and torch.equal(out[4], t[7])
    assert int(out[1].sum()) == 0 and int(out[3].sum()) == 0
