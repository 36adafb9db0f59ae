"""The native host library (plain C++, no CUDA): bulk file reads, Engram hashing,
row gathers and the paged-cache block allocator.  Built in-tree with g++ into ``_build/libdsv4_host.so`` and
bound with ctypes; :func:`lib` builds it on first use when the file is missing.
"""

from __future__ import annotations

import ctypes
import glob
import os
import subprocess
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
SRC = PKG / "csrc" / "host"
BUILD = PKG / "_build"
SO = BUILD / "libdsv4_host.so"
_lock = threading.Lock()
_lib = None


def sources() -> list[str]:
    return sorted(glob.glob(str(SRC / "*.cpp")))


def build(force: bool = False) -> Path:
    srcs = sources()
    newest = max(os.path.getmtime(s) for s in srcs)
    if SO.exists() and not force and os.path.getmtime(SO) >= newest:
        return SO
    BUILD.mkdir(parents=True, exist_ok=True)
    tmp = SO.with_suffix(f".{os.getpid()}.tmp")
    cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-pthread", "-fvisibility=hidden", "-march=x86-64-v2",
           *srcs, "-o", str(tmp)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    os.replace(tmp, SO)
    return SO


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(str(SO))
            i64p = ctypes.POINTER(ctypes.c_int64)
            L.dsv4_pread_many.argtypes = [ctypes.c_char_p, ctypes.c_int, i64p, i64p,
                                          ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]
            L.dsv4_pread_many.restype = ctypes.c_int
            _declare_engram(L)
            _declare_kv(L)
            _lib = L
    return _lib


def _declare_engram(L) -> None:
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    L.dsv4_engram_hash.argtypes = [vp, i64, vp, i64, vp, vp, vp, vp, vp]
    L.dsv4_engram_hash.restype = ctypes.c_int
    L.dsv4_gather_rows.argtypes = [vp, i64, i64, vp, i64, vp, ctypes.c_int]
    L.dsv4_gather_rows.restype = ctypes.c_int
    L.dsv4_fill_random.argtypes = [vp, i64, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.dsv4_fill_random.restype = ctypes.c_int


def _declare_kv(L) -> None:
    vp, c_int = ctypes.c_void_p, ctypes.c_int
    L.dsv4_kv_create.argtypes = [c_int, c_int, c_int]
    L.dsv4_kv_create.restype = vp
    L.dsv4_kv_destroy.argtypes = [vp]
    L.dsv4_kv_destroy.restype = None
    L.dsv4_kv_free_blocks.argtypes = [vp]
    L.dsv4_kv_free_blocks.restype = c_int
    L.dsv4_kv_slot_blocks.argtypes = [vp, c_int]
    L.dsv4_kv_slot_blocks.restype = c_int
    L.dsv4_kv_reserve.argtypes = [vp, c_int, c_int]
    L.dsv4_kv_reserve.restype = c_int
    L.dsv4_kv_release.argtypes = [vp, c_int]
    L.dsv4_kv_release.restype = None
    L.dsv4_kv_row.argtypes = [vp, c_int, vp]
    L.dsv4_kv_row.restype = None


class KvBlockAllocator:
    """Block pool + per-slot block table of one compression ratio (native,
    ``csrc/host/kv_blocks.cpp``)."""

    def __init__(self, n_blocks: int, n_slots: int, max_per_slot: int):
        self._L = lib()
        self._h = self._L.dsv4_kv_create(n_blocks, n_slots, max_per_slot)
        if not self._h:
            raise ValueError("invalid block allocator shape")
        self.n_blocks, self.n_slots, self.max_per_slot = n_blocks, n_slots, max_per_slot

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._L.dsv4_kv_destroy(h)
            self._h = None

    @property
    def free_blocks(self) -> int:
        return self._L.dsv4_kv_free_blocks(self._h)

    def slot_blocks(self, slot: int) -> int:
        return self._L.dsv4_kv_slot_blocks(self._h, slot)

    def reserve(self, slot: int, n_blocks: int) -> bool:
        """Grows ``slot`` to ``n_blocks`` blocks; False (nothing changed) when they do not fit."""
        return self._L.dsv4_kv_reserve(self._h, slot, n_blocks) == 0

    def release(self, slot: int) -> None:
        self._L.dsv4_kv_release(self._h, slot)

    def row(self, slot: int):
        """The slot's block ids (int32 numpy, -1 = unmapped)."""
        import numpy as np
        out = np.empty(self.max_per_slot, dtype=np.int32)
        self._L.dsv4_kv_row(self._h, slot, out.ctypes.data)
        return out


def fill_random(t, seed: int, mode: int, lo: int = 118, threads: int = 32) -> None:
    """Fills a contiguous uint8 host tensor: mode 0 = e4m3 codes (no NaN), 1 = ue8m0 bytes in [lo, lo+4]."""
    lib().dsv4_fill_random(t.data_ptr(), t.numel() * t.element_size(), seed, mode, lo, threads)


def engram_hash(hist, positions, mult, primes, offsets, pad: int, threads: int = 8):
    """Native twin of :meth:`..ref.engram.EngramHasher.hash` (numpy int64 arrays in and out)."""
    import numpy as np

    hist = np.ascontiguousarray(hist, dtype=np.int64)
    pos = np.ascontiguousarray(positions, dtype=np.int64)
    mult = np.ascontiguousarray(mult, dtype=np.int64)
    primes = np.ascontiguousarray(primes, dtype=np.int64)
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    nl, N = mult.shape
    H = primes.shape[-1]
    meta = np.array([nl, N, H, pad, threads], dtype=np.int64)
    out = np.empty((len(pos), nl, (N - 1) * H), dtype=np.int64)
    r = lib().dsv4_engram_hash(hist.ctypes.data, len(hist), pos.ctypes.data, len(pos), mult.ctypes.data,
                               primes.ctypes.data, offsets.ctypes.data, meta.ctypes.data, out.ctypes.data)
    if r != 0:
        raise ValueError(f"dsv4_engram_hash failed ({r})")
    return out


def gather_rows(table, ids, out=None, threads: int = 8):
    """out[i] = table[ids[i]] (rows of a 2-D host tensor), zero rows for out-of-range ids."""
    import numpy as np
    import torch

    ids = np.ascontiguousarray(ids, dtype=np.int64).reshape(-1)
    rb = table.shape[1] * table.element_size()
    if out is None:
        out = torch.empty((len(ids), table.shape[1]), dtype=table.dtype)
    lib().dsv4_gather_rows(table.data_ptr(), table.shape[0], rb, ids.ctypes.data, len(ids), out.data_ptr(), threads)
    return out


def pread_many(path: str, offsets: list[int], sizes: list[int], dst_ptrs: list[int], threads: int = 16) -> None:
    n = len(offsets)
    if n == 0:
        return
    A = ctypes.c_int64 * n
    P = ctypes.c_void_p * n
    r = lib().dsv4_pread_many(str(path).encode(), n, A(*offsets), A(*sizes), P(*dst_ptrs), threads)
    if r != 0:
        raise OSError(-r, f"pread_many failed on {path}: {os.strerror(-r)}")
