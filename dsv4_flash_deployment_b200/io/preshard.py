"""Pre-sharding: one contiguous, page-aligned blob per expert-parallel rank.

A rank of an EP=W deployment needs every dense tensor plus its own expert
range.  ``preshard`` writes ``rank{r}-of-{W}.bin`` (tensors at 4 KiB-aligned
offsets) with ``rank{r}-of-{W}.json`` (name -> dtype, shape, offset, nbytes,
and the blob's sha256).  ``load_shard`` reads a blob with the native threaded
reader into one pinned host buffer and, with ``device``, moves it to the GPU
in ONE copy; tensors are views into that allocation, so cold start is one
sequential read plus one H2D copy at link speed.

Reference: ``tpu-v7x/deepseek_v41/preshard.py:45-858`` (per-rank aligned
blobs) and ``load.py:347-735`` (mmap + mlock loader).
"""

from __future__ import annotations

import json
import re
from pathlib import Path

import torch

from .integrity import file_digest
from .safetensors import DTYPES, index_dir, read_tensors

ALIGN = 4096
_EXPERT = re.compile(r"\.ffn\.experts\.(\d+)\.")


def rank_tensor_names(names, n_experts_for_layer, rank: int, world: int) -> list[str]:
    """Dense tensors + this rank's contiguous expert range (per layer expert counts)."""
    out = []
    for n in names:
        m = _EXPERT.search(n)
        if m is None:
            out.append(n)
            continue
        layer = n.split(".ffn.")[0]
        e = int(m.group(1))
        per = n_experts_for_layer(layer) // world
        if rank * per <= e < (rank + 1) * per:
            out.append(n)
    return out


def preshard(ckpt_dir: str | Path, out_dir: str | Path, cfg, world: int, threads: int = 16) -> list[Path]:
    from .checkpoint_spec import checkpoint_specs

    idx = index_dir(ckpt_dir)
    specs = checkpoint_specs(cfg, include_mtp=False)
    names = [n for n in specs if n in idx]

    def n_exp(layer_prefix: str) -> int:
        lid = int(layer_prefix.split(".")[1])
        return cfg.n_experts_for(lid)

    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    written = []
    for r in range(world):
        sel = rank_tensor_names(names, n_exp, r, world)
        blob = out / f"rank{r}-of-{world}.bin"
        index, off = {}, 0
        with open(blob, "wb") as f:
            by_file: dict = {}
            for n in sel:
                by_file.setdefault(idx[n][0], []).append(n)
            for src, ns in by_file.items():
                ts = read_tensors(src, ns, threads=threads)
                for n in ns:
                    t = ts[n]
                    nb = t.numel() * t.element_size()
                    pad = (-off) % ALIGN
                    f.write(b"\0" * pad)
                    off += pad
                    f.write(t.contiguous().view(torch.uint8).reshape(-1).numpy().tobytes())
                    index[n] = {"dtype": idx[n][1].dtype, "shape": list(t.shape), "offset": off, "nbytes": nb}
                    off += nb
        meta = {"rank": r, "world": world, "model": cfg.name, "bytes": off, "sha256": file_digest(blob),
                "tensors": index}
        (out / f"rank{r}-of-{world}.json").write_text(json.dumps(meta))
        written.append(blob)
    return written


def load_shard(out_dir: str | Path, rank: int, world: int, device: str | torch.device | None = None,
               verify: bool = False, threads: int = 16) -> dict[str, torch.Tensor]:
    from ..ops.host import pread_many

    d = Path(out_dir)
    meta = json.loads((d / f"rank{rank}-of-{world}.json").read_text())
    blob = d / f"rank{rank}-of-{world}.bin"
    if verify:
        got = file_digest(blob)
        if got != meta["sha256"]:
            raise ValueError(f"{blob.name}: sha256 {got} != recorded {meta['sha256']}")
    nbytes = meta["bytes"]
    buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, pin_memory=torch.cuda.is_available())
    pread_many(str(blob), [0], [nbytes], [buf.data_ptr()], threads)
    if device is not None and torch.device(device).type == "cuda":
        dbuf = torch.empty_like(buf, device=device)
        dbuf.copy_(buf, non_blocking=True)
        torch.cuda.current_stream(torch.device(device)).synchronize()
        buf = dbuf
    out = {}
    for n, e in meta["tensors"].items():
        dt = DTYPES[e["dtype"]]
        o = e["offset"]
        out[n] = buf[o:o + e["nbytes"]].view(dt).reshape(e["shape"])
    return out
