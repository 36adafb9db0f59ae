"""Build and load the in-tree CUDA extension (sm_100a only).

``build()`` compiles every source under ``csrc/`` with nvcc for
``compute_100a/sm_100a`` (no other architecture) into
``dsv4_flash_deployment_b200/_build/dsv4_C.so``.  ``load()`` imports that file
directly; it never compiles, so a GPU box that received a pre-built tree only
loads it.  On a CUDA machine a missing extension is an error, not a fallback.

``DSV4_DEBUG_BOUNDS=1`` selects the debug-bounds variant (``dsv4_C_dbg`` in
``_build_dbg/``, compiled with ``-DDSV4_DEBUG_BOUNDS``): cache gathers and
writes check their indices and record a bad one in the device error word
instead of touching memory outside the buffer.  Build it with
``build(debug_bounds=True)``.
"""

from __future__ import annotations

import glob
import importlib.util
import os
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
NAME = "dsv4_C"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]

_mod = None

# kernels launched per binding call (used to report how many of this
# library's kernels a step issues)
_KERNELS_PER_CALL = {"hc_post": 1, "hc_finish": 1, "attention": 1, "gemm": 1, "gemm_a2": 1, "act_quant_mx": 1, "qkv_post": 1, "idx_q_prep": 1,
                     "compress_pool": 1, "ring_update": 1, "router_topk": 1, "router_small": 1, "moe_plan": 1, "moe_scatter": 1,
                     "indexer_topk": 2, "embed_streams": 1, "argmax_rows": 1, "act_roundtrip": 1,
                     "fp4_roundtrip": 1, "ep_pack": 1, "ep_unpack_meta": 1, "ep_unpack_rows": 1,
                     "ep_combine_pack": 1, "ep_wait": 1, "engram_gate": 1, "engram_prepare": 2,
                     "markov_step": 1, "tp_argmax_merge": 1}


class _Counting:
    """Proxy of the extension module that counts kernel launches."""

    def __init__(self, mod):
        self._mod = mod
        self.active = False
        self.count = 0

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        k = _KERNELS_PER_CALL.get(name)
        if k is None or not callable(fn):
            return fn

        def wrapped(*a, **kw):
            if self.active:
                n = k
                if name == "attention" and len(a) > 20 and a[20] > 1:
                    n = 2
                if name == "engram_prepare":
                    n = bin(int(a[18])).count("1")   # one kernel per mode bit (hash, ring, gather)
                self.count += n
            return fn(*a, **kw)

        return wrapped


class LaunchCounter:
    """Counts this library's kernel launches issued inside ``counting(True)``."""

    def __init__(self):
        self.count = 0

    def counting(self, on: bool):
        import contextlib

        @contextlib.contextmanager
        def cm():
            px = load()
            if not on or not isinstance(px, _Counting):
                yield
                return
            px.active, px.count = True, 0
            try:
                yield
            finally:
                px.active = False
                self.count = px.count

        return cm()


def sources() -> list[str]:
    return sorted(glob.glob(str(CSRC / "*.cu")) + glob.glob(str(CSRC / "*.cpp")))


def debug_bounds() -> bool:
    return os.environ.get("DSV4_DEBUG_BOUNDS", "0") == "1"


def _variant(dbg: bool) -> tuple[str, Path]:
    return (NAME + "_dbg", PKG / "_build_dbg") if dbg else (NAME, BUILD)


def so_path(dbg: bool | None = None) -> Path:
    name, d = _variant(debug_bounds() if dbg is None else dbg)
    return d / f"{name}.so"


def build(verbose: bool = False, debug_bounds: bool = False):
    """Compile the extension in-tree (works without a GPU)."""
    from torch.utils import cpp_extension

    name, bdir = _variant(debug_bounds)
    bdir.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(max(1, (os.cpu_count() or 4))))
    extra = ["-DDSV4_DEBUG_BOUNDS"] if debug_bounds else []
    mod = cpp_extension.load(
        name=name,
        sources=sources(),
        extra_cflags=CXX_FLAGS + extra,
        extra_cuda_cflags=NVCC_FLAGS + extra,
        extra_include_paths=[str(CSRC)],
        build_directory=str(bdir),
        verbose=verbose,
        with_cuda=True,
    )
    return mod


def load(required: bool | None = None):
    """Import the pre-built extension; raise if it is required and missing."""
    global _mod
    if _mod is not None:
        return _mod
    import torch  # noqa: F401  (the extension links against torch)

    path = so_path()
    if required is None:
        required = torch.cuda.is_available()
    if not path.exists():
        if required:
            raise RuntimeError(f"CUDA extension not built: {path} missing (run __graft_entry__.build())")
        return None
    name = path.stem
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    _mod = _Counting(mod)
    return _mod
