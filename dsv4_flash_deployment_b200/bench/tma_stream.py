"""Builds and runs the TMA / bulk-copy streaming probe (``tma_stream_probe.cu``).

The probe measures the read bandwidth one CTA per SM reaches when it streams a
4 GB matrix into shared memory through 2-D tensor tiles (the GEMM weight path)
or 1-D bulk copies, in several access orders and stage shapes.  It is the
denominator against which the GEMMs' weight streaming is judged (a plain copy
also writes, so read-only streaming can exceed the measured copy bandwidth).

    python -m dsv4_flash_deployment_b200.bench.tma_stream
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE.parent / "_build"


def build() -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    exe = BUILD / "tma_stream_probe"
    src = HERE / "tma_stream_probe.cu"
    if not exe.exists() or exe.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", str(src), "-lcuda",
                        "-o", str(exe)], check=True)
    return exe


def main() -> None:
    exe = build()
    raise SystemExit(subprocess.run([str(exe)]).returncode)


if __name__ == "__main__":
    main()
