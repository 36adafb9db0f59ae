"""Random-init Engram tables in shared files (one copy per node): the first
process fills a table, later ones map the same pages, a changed shape or seed
rebuilds it, and concurrent processes fill it exactly once (CPU only)."""

import os
import subprocess
import sys

import torch

from dsv4_flash_deployment_b200.models.engram import shared_table
from dsv4_flash_deployment_b200.ops import host


def _filler(seed, calls):
    def fill(t):
        calls.append(seed)
        host.fill_random(t, seed, 0)
    return fill


def test_first_process_fills_later_ones_map(tmp_path):
    prefix = str(tmp_path / "eng")
    calls = []
    a = shared_table(prefix, "l1.q", 1000, 64, _filler(7, calls), "e4m3 seed 7")
    ref = torch.empty(1000, 64, dtype=torch.uint8)
    host.fill_random(ref, 7, 0)
    assert torch.equal(a, ref) and calls == [7]
    b = shared_table(prefix, "l1.q", 1000, 64, _filler(7, calls), "e4m3 seed 7")
    assert torch.equal(b, ref) and calls == [7]          # mapped, not refilled
    b[0, 0] ^= 1                                          # one set of pages behind both views
    assert a[0, 0] == b[0, 0]
    c = shared_table(prefix, "l1.q", 1000, 64, _filler(8, calls), "e4m3 seed 8")
    assert calls == [7, 8] and not torch.equal(c, ref)    # another signature rebuilds
    d = shared_table(prefix, "l1.q", 500, 64, _filler(8, calls), "e4m3 seed 8")
    assert calls == [7, 8, 8] and d.shape == (500, 64)    # another shape rebuilds
    assert os.path.getsize(prefix + ".l1.q") == 500 * 64


_CHILD = """
import sys, torch
from dsv4_flash_deployment_b200.models.engram import shared_table
from dsv4_flash_deployment_b200.ops import host
filled = []
t = shared_table(sys.argv[1], "l14.sf", 200000, 8, lambda x: (filled.append(1), host.fill_random(x, 3, 1, 118)),
                 "ue8m0 seed 3")
print(len(filled), int(t.to(torch.int64).sum()))
"""


def test_concurrent_processes_fill_once(tmp_path):
    prefix = str(tmp_path / "eng")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
    procs = [subprocess.Popen([sys.executable, "-c", _CHILD, prefix], stdout=subprocess.PIPE, text=True, env=env)
             for _ in range(3)]
    outs = [p.communicate(timeout=300)[0].split() for p in procs]
    assert all(p.returncode == 0 for p in procs)
    assert sum(int(o[0]) for o in outs) == 1              # exactly one process filled
    assert len({o[1] for o in outs}) == 1                 # all saw the same bytes


def test_shared_tables_must_be_page_lockable(monkeypatch):
    """The GPU page-locks the shared mapping: tmpfs / hugetlbfs prefixes pass, a
    regular file system is refused up front with the reason."""
    import pytest

    from dsv4_flash_deployment_b200.models import engram as E

    monkeypatch.setattr(E, "mount_fs_type", lambda p: "ext4")
    with pytest.raises(ValueError, match="tmpfs"):
        E.check_page_lockable("/somewhere/engram")
    monkeypatch.setattr(E, "mount_fs_type", lambda p: "tmpfs")
    E.check_page_lockable("/dev/shm/engram")
    monkeypatch.setattr(E, "mount_fs_type", lambda p: None)      # unknown: not refused
    E.check_page_lockable("/x/engram")
