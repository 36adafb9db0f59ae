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


class _FakeRegistry:
    """Stands in for the extension's page-locking calls: a registered range reports
    is_pinned(), as cudaHostRegister'd memory does."""

    def __init__(self):
        self.live = {}
        self.calls = []

    def host_register(self, addr, nbytes):
        assert addr not in self.live, "range registered twice"
        self.live[addr] = nbytes
        self.calls.append(("register", addr))
        return addr + (1 << 40)

    def host_unregister(self, addr):
        del self.live[addr]
        self.calls.append(("unregister", addr))

    def host_device_ptr(self, addr):
        return addr + (1 << 40)


def test_host_table_registration_outlives_every_user(monkeypatch):
    # two models over the same weight tensors: the second table sees a range the
    # first registered (is_pinned() True) and must still count as a user, so that
    # freeing the first model leaves the range registered for the second
    from dsv4_flash_deployment_b200.models.engram import HostTable

    fake = _FakeRegistry()
    monkeypatch.setattr(torch.Tensor, "is_pinned",
                        lambda self, *a: self.untyped_storage().data_ptr() in fake.live)
    monkeypatch.setattr(HostTable, "_registered", {})
    q = torch.randint(0, 255, (64, 64), dtype=torch.uint8)
    sf = torch.randint(118, 123, (64, 2), dtype=torch.uint8)
    first = HostTable(q, sf, fake)
    second = HostTable(q, sf, fake)
    assert second.dq == first.dq and second.dsf == first.dsf
    assert [c for c, _ in fake.calls] == ["register", "register"]
    first.release(fake)
    assert set(fake.live) == {q.untyped_storage().data_ptr(), sf.untyped_storage().data_ptr()}
    second.release(fake)
    assert fake.live == {}


def test_host_table_uses_caller_pinned_memory_as_is(monkeypatch):
    from dsv4_flash_deployment_b200.models.engram import HostTable

    fake = _FakeRegistry()
    monkeypatch.setattr(torch.Tensor, "is_pinned", lambda self, *a: True)
    monkeypatch.setattr(HostTable, "_registered", {})
    q = torch.zeros(8, 64, dtype=torch.uint8)
    t = HostTable(q, torch.zeros(8, 2, dtype=torch.uint8), fake)
    assert fake.calls == [] and t.storages == []
    assert t.dq == q.data_ptr() + (1 << 40)
