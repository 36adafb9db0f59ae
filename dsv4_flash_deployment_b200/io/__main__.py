"""Checkpoint tools from the command line.

    python -m dsv4_flash_deployment_b200.io synth    --model v4.1-tiny --out ckpt/ [--seed 0] [--shard-gib 4] [--mtp]
    python -m dsv4_flash_deployment_b200.io inspect  --model v4.1-flash --ckpt ckpt/ [--mtp]
    python -m dsv4_flash_deployment_b200.io manifest --ckpt ckpt/
    python -m dsv4_flash_deployment_b200.io verify   --ckpt ckpt/
    python -m dsv4_flash_deployment_b200.io preshard --model v4.1-flash --ckpt ckpt/ --out shards/ --world 8

``synth`` writes a random-weight checkpoint of a named model in the checkpoint
layout (sharded safetensors plus an integrity manifest), the counterpart of the
reference's synthetic checkpoint writer (``tpu-v7x/deepseek_v41/checkpoint.py``
``write_synthetic_checkpoint`` ``:295``).  ``inspect`` checks a checkpoint
against the model's tensor specification and reports every missing, unexpected
or mismatched tensor (the reference's loader fails loudly on unfilled
parameters, ``P/0005:1078``) and exits non-zero if any is missing or
mismatched.  ``manifest`` / ``verify`` write and check the per-file sha256
manifest (the reference verifies recorded checkpoint hashes before loading,
``megakernel/load.py:39``).  ``preshard`` writes one page-aligned blob per
expert-parallel rank (``io/preshard.py``).  Each command prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import sys
import time


def _cfg(name: str):
    from ..config import ModelConfig, get_config

    return ModelConfig.from_json(name) if name.endswith(".json") else get_config(name)


def cmd_synth(a) -> dict:
    from .checkpoint_spec import make_random_weights
    from .integrity import write_manifest
    from .safetensors import save_checkpoint

    cfg = _cfg(a.model)
    t0 = time.perf_counter()
    w = make_random_weights(cfg, seed=a.seed, include_mtp=a.mtp)
    files = save_checkpoint(a.out, w, cfg, shard_bytes=int(a.shard_gib * 2 ** 30))
    write_manifest(a.out)
    nbytes = sum(t.numel() * t.element_size() for t in w.values())
    return {"out": a.out, "model": cfg.name, "tensors": len(w), "bytes": nbytes, "files": len(files),
            "seconds": round(time.perf_counter() - t0, 2)}


def inspect(ckpt: str, cfg, include_mtp: bool) -> dict:
    from .checkpoint_spec import checkpoint_specs
    from .safetensors import index_dir

    specs = checkpoint_specs(cfg, include_mtp=include_mtp)
    idx = index_dir(ckpt)
    missing = sorted(n for n in specs if n not in idx)
    unexpected = sorted(n for n in idx if n not in specs)
    mismatched = []
    dtypes: dict[str, int] = {}
    nbytes = 0
    for n, (f, e) in idx.items():
        dtypes[e.dtype] = dtypes.get(e.dtype, 0) + 1
        nbytes += e.nbytes
        if n in specs:
            tag, shape = specs[n]
            ok_tag = e.dtype == tag or (tag == "F8_E8M0" and e.dtype in ("U8", "F8_E8M0")) or \
                (tag == "I8" and e.dtype in ("I8", "U8"))
            if not ok_tag or tuple(e.shape) != tuple(shape):
                mismatched.append(f"{n}: {e.dtype}{list(e.shape)} != {tag}{list(shape)}")
    return {"ckpt": str(ckpt), "model": cfg.name, "tensors": len(idx), "expected": len(specs),
            "bytes": nbytes, "dtypes": dtypes, "missing": len(missing), "unexpected": len(unexpected), "mismatched": len(mismatched),
            "first_missing": missing[:10], "first_unexpected": unexpected[:10], "first_mismatched": mismatched[:10],
            "ok": not missing and not mismatched}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m dsv4_flash_deployment_b200.io", description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("synth")
    s.add_argument("--model", required=True)
    s.add_argument("--out", required=True)
    s.add_argument("--seed", type=int, default=0)
    s.add_argument("--shard-gib", type=float, default=4.0)
    s.add_argument("--mtp", action="store_true", help="include the DSpark MTP stages")
    i = sub.add_parser("inspect")
    i.add_argument("--model", required=True)
    i.add_argument("--ckpt", required=True)
    i.add_argument("--mtp", action="store_true")
    m = sub.add_parser("manifest")
    m.add_argument("--ckpt", required=True)
    v = sub.add_parser("verify")
    v.add_argument("--ckpt", required=True)
    p = sub.add_parser("preshard")
    p.add_argument("--model", required=True)
    p.add_argument("--ckpt", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--world", type=int, required=True)
    a = ap.parse_args(argv)
    rc = 0
    if a.cmd == "synth":
        out = cmd_synth(a)
    elif a.cmd == "inspect":
        out = inspect(a.ckpt, _cfg(a.model), a.mtp)
        rc = 0 if out["ok"] else 1
    elif a.cmd == "manifest":
        from .integrity import write_manifest

        out = {"manifest": str(write_manifest(a.ckpt))}
    elif a.cmd == "verify":
        from .integrity import IntegrityError, verify_manifest

        try:
            out = {"ok": True, **verify_manifest(a.ckpt)}
        except (IntegrityError, FileNotFoundError) as e:
            out, rc = {"ok": False, "error": str(e)}, 1
    else:
        from .preshard import preshard

        t0 = time.perf_counter()
        files = preshard(a.ckpt, a.out, _cfg(a.model), a.world)
        out = {"files": [str(f) for f in files], "seconds": round(time.perf_counter() - t0, 2)}
    print(json.dumps(out))
    return rc


if __name__ == "__main__":
    sys.exit(main())
