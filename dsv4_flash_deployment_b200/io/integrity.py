"""Checkpoint integrity: per-file sha256 manifests, verified before loading.

The reference verifies checkpoint files against recorded hashes before it
loads them (``megakernel-recipe/megakernel/load.py:39``,
``results/ckpt_hashes.json``); a corrupt or truncated shard fails loudly.
"""

from __future__ import annotations

import hashlib
import json
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

MANIFEST = "checkpoint_sha256.json"


def file_digest(path: str | Path, chunk: int = 16 << 20) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(chunk)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def _files(d: Path) -> list[Path]:
    return sorted(p for p in d.iterdir() if p.is_file() and p.suffix in (".safetensors", ".bin", ".json")
                  and p.name != MANIFEST)


def write_manifest(ckpt_dir: str | Path, threads: int = 8) -> Path:
    d = Path(ckpt_dir)
    files = _files(d)
    with ThreadPoolExecutor(threads) as ex:
        digests = list(ex.map(file_digest, files))
    m = {f.name: {"sha256": h, "bytes": f.stat().st_size} for f, h in zip(files, digests)}
    out = d / MANIFEST
    out.write_text(json.dumps(m, indent=1))
    return out


class IntegrityError(ValueError):
    pass


def verify_manifest(ckpt_dir: str | Path, threads: int = 8) -> dict:
    d = Path(ckpt_dir)
    m = json.loads((d / MANIFEST).read_text())
    names = sorted(m)
    for n in names:
        if not (d / n).exists():
            raise IntegrityError(f"{n}: listed in the manifest but missing")
    with ThreadPoolExecutor(threads) as ex:
        got = dict(zip(names, ex.map(lambda n: file_digest(d / n), names)))
    bad = [n for n in names if got[n] != m[n]["sha256"]]
    if bad:
        raise IntegrityError(f"sha256 mismatch in {len(bad)} file(s): {bad[:5]}")
    return {"files": len(names), "bytes": sum(v["bytes"] for v in m.values())}
