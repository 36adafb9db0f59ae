"""The native host library (plain C++, no CUDA): bulk file reads, Engram hashing
and row gathers.  Built in-tree with g++ into ``_build/libdsv4_host.so`` and
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
            _lib = L
    return _lib


def _declare_engram(L) -> None:
    if not hasattr(L, "dsv4_engram_hash"):
        return
    i64p = ctypes.POINTER(ctypes.c_int64)
    L.dsv4_engram_hash.argtypes = [i64p, ctypes.c_int64, i64p, ctypes.c_int64, i64p, ctypes.c_int, ctypes.c_int,
                                   i64p, i64p, ctypes.c_int64, i64p]
    L.dsv4_engram_hash.restype = ctypes.c_int
    if hasattr(L, "dsv4_gather_rows"):
        L.dsv4_gather_rows.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, i64p, ctypes.c_int64,
                                       ctypes.c_void_p, ctypes.c_int]
        L.dsv4_gather_rows.restype = ctypes.c_int


def pread_many(path: str, offsets: list[int], sizes: list[int], dst_ptrs: list[int], threads: int = 16) -> None:
    n = len(offsets)
    if n == 0:
        return
    A = ctypes.c_int64 * n
    P = ctypes.c_void_p * n
    r = lib().dsv4_pread_many(str(path).encode(), n, A(*offsets), A(*sizes), P(*dst_ptrs), threads)
    if r != 0:
        raise OSError(-r, f"pread_many failed on {path}: {os.strerror(-r)}")
