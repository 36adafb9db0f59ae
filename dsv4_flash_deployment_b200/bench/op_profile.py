"""Per-op time breakdown of one model step, from CUDA events (no profiler).

Builds the same V4-Flash steady-state step as ``bench.py`` (or a smaller
config), runs it eagerly with event pairs around every op group, and prints
milliseconds per step per group plus the share of the step.

    python -m dsv4_flash_deployment_b200.bench.op_profile [--steps 3]
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from ..config import v4_flash_config
from ..engine.engine import Engine
from ..engine.memory import plan_expert_storage
from ..models.model import SeqChunk, StepMeta


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--concurrency", type=int, default=512)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--layers", type=int, default=None, help="override n_layers (smaller smoke runs)")
    ap.add_argument("--experts", type=int, default=None, help="override routed experts (small profiling cases)")
    ap.add_argument("--topk", type=int, default=None)
    ap.add_argument("--ep-transport", default="p2p", choices=["p2p", "nccl"])
    ap.add_argument("--decode-only", action="store_true", help="C decoding sequences per rank, no prefill chunk")
    ap.add_argument("--context", type=int, default=1024, help="decode positions start here (span of 1024)")
    a = ap.parse_args()
    import os

    import torch.distributed as dist

    from ..parallel.ep import EPGroup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    ep = None
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        ep = EPGroup(rank, world, dist.group.WORLD, torch.device("cuda", local), transport=a.ep_transport)
    kw = {"n_layers": a.layers} if a.layers else {}
    if a.experts:
        kw["n_routed_experts"] = a.experts
    if a.topk:
        kw["n_activated_experts"] = a.topk
    cfg = v4_flash_config(**kw)
    dev = torch.device("cuda", local)
    n_dec = a.concurrency // world - (0 if a.decode_only else 1)
    chunk = 0 if a.decode_only else a.chunk // world
    T = n_dec + chunk
    max_seq = a.context + 1024 + 16
    n_phys = plan_expert_storage(cfg, dev, T, n_dec + 2, max_seq, world)
    eng = Engine.build(cfg, dev, max_seqs=n_dec + 2, max_batched_tokens=T, max_seq_len=max_seq,
                       expert_storage_layers=n_phys, use_graphs=False, ep=ep)
    m = eng.model
    rng = np.random.default_rng(0)
    dec = a.context + (np.arange(n_dec) * (1024 // max(1, n_dec)) + 1) % 1024

    def meta(i):
        ch = [SeqChunk(s, int(dec[s]) + i, [int(rng.integers(0, cfg.vocab_size))], True) for s in range(n_dec)]
        if chunk:
            ch.append(SeqChunk(n_dec, (i % 2) * chunk, rng.integers(0, cfg.vocab_size, chunk).tolist(), i % 2 == 1))
        return StepMeta(cfg, ch)

    eng.run_meta(meta(0))
    m.op_timer = {}
    tot_s, tot_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    tot_s.record()
    for i in range(a.steps):
        mm = meta(i + 1)
        m.upload(mm)
        m.forward(mm)
    tot_e.record()
    torch.cuda.synchronize()
    total = tot_s.elapsed_time(tot_e) / a.steps
    rows = {k: sum(s.elapsed_time(e) for s, e in v) / a.steps for k, v in m.op_timer.items()}
    acc = sum(rows.values())
    if rank == 0:
        for k, v in sorted(rows.items(), key=lambda x: -x[1]):
            print(f"{k:20s} {v:9.3f} ms  {100 * v / total:5.1f}%  ({len(m.op_timer[k]) // a.steps} launches/step)")
        print(json.dumps({"step_ms": round(total, 3), "sum_ops_ms": round(acc, 3), "T": T, "n_layers": cfg.n_layers,
                          "expert_storage_layers": n_phys, "world": world}))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
