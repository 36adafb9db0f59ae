"""Engram on the device, with the embedding tables in pinned host memory.

V4.1 adds, before the blocks of layers 1 and 14, a lookup of 24 hashed
n-gram rows (orders 2..4 x 8 heads) per token in two ~100 GB FP8 tables, an
FP8 ``wkv`` projection to 4 keys + 1 value, and a per-stream sigmoid gate
(``reference.py:272-319``; host-resident tables in the vLLM recipe,
P/0005:1183-1370).  Here:

* the tables stay in page-locked host memory (``cudaHostRegister`` of the
  loaded arrays, of pinned allocations for random init, or of shared files
  under ``/dev/shm`` that every rank of the node maps, as the reference keeps
  its tables in ``/dev/shm``: ``MK/megakernel/load.py:203-355``) and the GPU reads the
  rows it needs straight over the host link: 24 x (256 + 8) bytes per token
  and layer, with no host thread on the step's critical path;
* hashing runs on the GPU from this step's tokens and a per-slot ring of the
  previous 3 compressed ids (the int64 contract of ``ref/engram.py``);
* the gathered rows are already MXFP8 (e4m3 + ue8m0 per 32), so they feed the
  block-scaled tcgen05 GEMM directly as its A operand; a small kernel applies
  the gate to the four residual streams.

Hash + gather for every Engram layer run once per step at the first Engram
layer; each Engram layer then runs its GEMM and gate.
"""

from __future__ import annotations

import numpy as np
import torch

from ..ops.gemm import MxWeight
from ..ops.layout import ceil_to, expand_block_scales
from ..ref.engram import EngramHasher


PAGE_LOCKABLE_FS = ("tmpfs", "hugetlbfs")


def mount_fs_type(path: str) -> str | None:
    """File system type of the mount that holds ``path`` (from ``/proc/mounts``),
    or None where that is unknown."""
    import os

    p = os.path.realpath(path)
    best, typ = "", None
    try:
        with open("/proc/mounts") as f:
            for line in f:
                parts = line.split()
                if len(parts) < 3:
                    continue
                mnt = parts[1].replace("\\040", " ")
                inside = p == mnt or p.startswith(mnt.rstrip("/") + "/")
                if inside and len(mnt) >= len(best):
                    best, typ = mnt, parts[2]
    except OSError:
        return None
    return typ


def check_page_lockable(prefix: str) -> None:
    """Shared table files must sit on tmpfs (``/dev/shm``) or hugetlbfs: Linux
    refuses long-term pinning of writable shared mappings of regular files, so
    ``cudaHostRegister`` of such a mapping fails ("invalid argument")."""
    import os

    d = os.path.dirname(os.path.abspath(prefix)) or "."
    typ = mount_fs_type(d)
    if typ is not None and typ not in PAGE_LOCKABLE_FS:
        raise ValueError(f"Engram shared tables at {prefix!r} are on a {typ} file system; the GPU reads them "
                         f"from page-locked memory, which needs tmpfs or hugetlbfs (e.g. /dev/shm/<name>)")


def shared_table(prefix: str, tag: str, rows: int, width: int, fill, signature: str) -> torch.Tensor:
    """uint8 [rows, width] backed by the shared file ``<prefix>.<tag>`` (e.g. under
    ``/dev/shm``), filled once for all processes.

    The first process to take the file's lock creates and fills it and then writes
    a ``.ready`` marker holding the shape and ``signature`` (the fill's seed and
    mode); every later process (the other ranks of the node, or a restarted
    server) maps the same pages without filling.  A marker for another shape or
    signature makes the next process rebuild the file.  The files outlive the
    processes; delete them to free the memory.
    """
    import fcntl
    import json
    import os

    path = f"{prefix}.{tag}"
    nbytes = rows * width
    sig = json.dumps({"rows": rows, "width": width, "fill": signature})
    with open(path + ".lock", "a") as lk:
        fcntl.flock(lk, fcntl.LOCK_EX)
        try:
            ready = path + ".ready"
            ok = (os.path.exists(ready) and os.path.exists(path) and os.path.getsize(path) == nbytes
                  and open(ready).read() == sig)
            if not ok:
                for f in (ready, path):
                    if os.path.exists(f):
                        os.remove(f)
                t = torch.from_file(path, shared=True, size=nbytes, dtype=torch.uint8)
                fill(t.view(rows, width))
                with open(ready, "w") as f:
                    f.write(sig)
            else:
                t = torch.from_file(path, shared=True, size=nbytes, dtype=torch.uint8)
        finally:
            fcntl.flock(lk, fcntl.LOCK_UN)
    return t.view(rows, width)


class HostTable:
    """One layer's table: e4m3 rows [n_emb, hd] + ue8m0 scales [n_emb, hd/32], page-locked.

    Pageable tensors are page-locked in place by registering their whole
    storage once (tensors loaded from one checkpoint file share a storage, and
    two registrations may not overlap); pinned tensors are used as they are.
    """

    _registered: dict[int, tuple[int, int]] = {}   # storage address -> (device address, users)

    def __init__(self, q: torch.Tensor, sf: torch.Tensor, ext):
        self.q, self.sf = q.contiguous().view(torch.uint8), sf.contiguous().view(torch.uint8)
        self.n = self.q.shape[0]
        self._ext = ext
        self.storages = []
        self.dq = self._device_addr(self.q, ext)
        self.dsf = self._device_addr(self.sf, ext)

    def _device_addr(self, t: torch.Tensor, ext) -> int:
        st = t.untyped_storage()
        base = st.data_ptr()
        # our own registrations first: a registered range also reports is_pinned(),
        # and a table that took it as pinned memory would hold no user count, so
        # the release of another table over the same storage (a second model
        # built from the same weights) would unregister it under this one
        reg = HostTable._registered.get(base)
        if reg is None:
            if t.is_pinned():
                return int(ext.host_device_ptr(base)) + (t.data_ptr() - base)
            reg = (int(ext.host_register(base, st.nbytes())), 0)
        HostTable._registered[base] = (reg[0], reg[1] + 1)
        self.storages.append(base)
        return reg[0] + (t.data_ptr() - base)

    def __del__(self):
        # a registration must not outlive its storage (a freed, still-registered
        # range makes later copies through reused memory fail)
        try:
            if self.storages:
                self.release(self._ext)
        except Exception:
            pass

    def release(self, ext) -> None:
        for base in self.storages:
            dev, users = HostTable._registered[base]
            if users <= 1:
                ext.host_unregister(base)
                del HostTable._registered[base]
            else:
                HostTable._registered[base] = (dev, users - 1)
        self.storages = []


class EngramRuntime:
    def __init__(self, cfg, dev, n_slots: int, max_tokens: int, ext, weights: dict | None = None, seed: int = 0,
                 shm_prefix: str | None = None, token_map=None):
        """``shm_prefix`` (random init only): keep the tables in shared files
        ``<shm_prefix>.l<layer>.{q,sf}`` that every process of the node maps (one
        copy per node instead of one per rank; see :func:`shared_table`).
        ``token_map``: token id -> compressed id (``ref.engram.compressed_token_map``
        of the checkpoint's tokenizer); None: ``id % C``."""
        self.cfg, self.dev, self.ext = cfg, dev, ext
        if shm_prefix and weights is None:
            check_page_lockable(shm_prefix)
        h = EngramHasher(cfg, token_map=token_map)
        lay = h.layout
        self.nl, self.N, self.H, self.hd = len(lay.layer_ids), lay.max_ngram, lay.n_heads, lay.head_dim
        self.cols = (self.N - 1) * self.H
        self.K = self.cols * self.hd
        i64 = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.int64, device=dev)
        self.token_map = i64(h.token_map)
        self.mult, self.primes, self.offsets = i64(h.mult), i64(lay.primes), i64(lay.offsets)
        self.pad = int(h.pad)
        self.ring = torch.zeros(n_slots, self.N - 1, dtype=torch.int64, device=dev)
        self.rows = torch.zeros(max_tokens, self.nl, self.cols, dtype=torch.int64, device=dev)
        tp = ceil_to(max_tokens, 128)
        self.a_q = torch.zeros(self.nl, tp, self.K, dtype=torch.uint8, device=dev)
        self.a_sf = torch.full((self.nl, (tp // 128) * (self.K // 128) * 512), 127, dtype=torch.uint8, device=dev)
        D, hc = cfg.dim, cfg.hc_mult
        self.kv = torch.empty(max_tokens, (hc + 1) * D, dtype=torch.bfloat16, device=dev)
        self.layer_index = {lid: i for i, lid in enumerate(lay.layer_ids)}
        self.tables, self.wkv, self.wgt = [], [], []
        g = torch.Generator().manual_seed(seed + 4242)
        for i, lid in enumerate(lay.layer_ids):
            p = f"layers.{lid}.engram"
            if weights is not None:
                q, sf = weights[f"{p}.embed.weight"], weights[f"{p}.embed.scale"]
                wkv = MxWeight.from_checkpoint(weights[f"{p}.wkv.weight"],
                                               expand_block_scales(weights[f"{p}.wkv.scale"],
                                                                   weights[f"{p}.wkv.weight"].shape[0]), dev)
                qw, kw = weights[f"{p}.q_weight"], weights[f"{p}.k_weight"]
            else:
                # tables of the full model are ~100 GB each: fill them with the native
                # multithreaded generator, then page-lock them in place (HostTable)
                from ..ops import host
                n_emb = lay.num_embeddings[i]
                sq, ssf = seed * 1000 + 2 * i + 1, seed * 1000 + 2 * i + 2
                if shm_prefix:
                    q = shared_table(shm_prefix, f"l{lid}.q", n_emb, self.hd,
                                     lambda t, s=sq: host.fill_random(t, s, 0), f"e4m3 seed {sq}")
                    sf = shared_table(shm_prefix, f"l{lid}.sf", n_emb, self.hd // 32,
                                      lambda t, s=ssf: host.fill_random(t, s, 1, 118), f"ue8m0 seed {ssf} lo 118")
                else:
                    q = torch.empty(n_emb, self.hd, dtype=torch.uint8)
                    sf = torch.empty(n_emb, self.hd // 32, dtype=torch.uint8)
                    host.fill_random(q, sq, 0)
                    host.fill_random(sf, ssf, 1, 118)
                wq = (torch.randn((hc + 1) * D, self.K, generator=g) * 0.5).to(torch.float8_e4m3fn)
                ws = torch.randint(118, 123, ((hc + 1) * D // 32, self.K // 32), generator=g,
                                   dtype=torch.int32).to(torch.uint8)
                wkv = MxWeight.from_checkpoint(wq, expand_block_scales(ws, (hc + 1) * D), dev)
                qw = (1 + 0.05 * torch.randn(hc, D, generator=g)).to(torch.bfloat16)
                kw = (1 + 0.05 * torch.randn(hc, D, generator=g)).to(torch.bfloat16)
            self.tables.append(HostTable(q, sf, ext))
            self.wkv.append(wkv)
            self.wgt.append((qw.float() * kw.float()).to(dev).contiguous())
        self.table_addrs = torch.tensor([[t.dq, t.dsf, t.n] for t in self.tables], dtype=torch.int64)

    def prepare(self, model, T: int, update_ring: bool = True) -> None:
        """Hashes this step's tokens and gathers every Engram layer's rows from host memory.

        ``update_ring=False`` (speculative verify) leaves the token ring untouched;
        :meth:`commit_ring` then stores only the accepted tokens.
        """
        self.ext.engram_prepare(model.m_ids, model.m_pos, model.m_slot, model.m_cstart, model.m_row0, model.m_last,
                                T, self.token_map, self.ring, self.mult, self.primes, self.offsets, self.pad,
                                self.rows, self.table_addrs, self.a_q, self.a_sf, self.hd, 7 if update_ring else 5)

    def commit_ring(self, model, T: int, last_pos: torch.Tensor) -> None:
        """Stores the ring tokens of positions <= last_pos (per token) from the last step's ids."""
        self.ext.engram_prepare(model.m_ids, model.m_pos, model.m_slot, model.m_cstart, model.m_row0, last_pos,
                                T, self.token_map, self.ring, self.mult, self.primes, self.offsets, self.pad,
                                self.rows, None, None, None, self.hd, 2)

    def apply(self, model, lid: int, T: int) -> None:
        """X += gate * value for Engram layer ``lid`` (rows gathered by :meth:`prepare`)."""
        i = self.layer_index[lid]
        model._gemm(self.a_q[i], self.a_sf[i], T, self.wkv[i], self.kv)
        self.ext.engram_gate(model.X, self.kv, self.wgt[i], T, self.cfg.rms_norm_eps)

    def release(self) -> None:
        for t in self.tables:
            t.release(self.ext)
