"""Build and load the in-tree CUDA extension (sm_100a only).

``build()`` compiles every source under ``csrc/`` with nvcc for
``compute_100a/sm_100a`` (no other architecture) into
``dsv4_flash_deployment_b200/_build/dsv4_C.so``.  ``load()`` imports that file
directly; it never compiles, so a GPU box that received a pre-built tree only
loads it.  On a CUDA machine a missing extension is an error, not a fallback.
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


def sources() -> list[str]:
    return sorted(glob.glob(str(CSRC / "*.cu")) + glob.glob(str(CSRC / "*.cpp")))


def so_path() -> Path:
    return BUILD / f"{NAME}.so"


def build(verbose: bool = False):
    """Compile the extension in-tree (works without a GPU)."""
    from torch.utils import cpp_extension

    BUILD.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(max(1, (os.cpu_count() or 4))))
    mod = cpp_extension.load(
        name=NAME,
        sources=sources(),
        extra_cflags=CXX_FLAGS,
        extra_cuda_cflags=NVCC_FLAGS,
        extra_include_paths=[str(CSRC)],
        build_directory=str(BUILD),
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
    spec = importlib.util.spec_from_file_location(NAME, str(path))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[NAME] = mod
    spec.loader.exec_module(mod)
    _mod = mod
    return mod
