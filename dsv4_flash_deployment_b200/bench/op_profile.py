"""Per-op time breakdown of one model step (no profiler).

Builds the same V4-Flash steady-state step as ``bench.py`` (or a smaller
config) and prints milliseconds per step per op group plus the share of the
step.  Two ways to time it:

* default: eager steps with CUDA-event pairs around every op group (host
  launch gaps of eager mode are included);
* ``--device-trace``: the step is captured in a CUDA graph with a device
  timestamp mark after every op group (``utils/devtrace.py``) and replayed;
  works under ``torchrun`` (every rank traces; the table shows the max over
  ranks of each group and the untraced graph step time for comparison).

    python -m dsv4_flash_deployment_b200.bench.op_profile [--steps 3]
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m dsv4_flash_deployment_b200.bench.op_profile \
        --device-trace --steps 5
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
    ap.add_argument("--family", default="v4", choices=["v4", "v41"],
                    help="v4: the V4-Flash-shaped model; v41: the V4.1-Flash architecture (Engram, MXFP4 experts)")
    ap.add_argument("--engram-rows", type=int, default=4_000_000, help="v41: rows per Engram table")
    ap.add_argument("--concurrency", type=int, default=512)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--layers", type=int, default=None, help="override n_layers (smaller smoke runs)")
    ap.add_argument("--experts", type=int, default=None, help="override routed experts (small profiling cases)")
    ap.add_argument("--topk", type=int, default=None)
    ap.add_argument("--ep-transport", default="fused", choices=["p2p", "nccl", "fused"])
    ap.add_argument("--decode-only", action="store_true", help="C decoding sequences per rank, no prefill chunk")
    ap.add_argument("--context", type=int, default=1024, help="decode positions start here (span of 1024)")
    ap.add_argument("--device-trace", action="store_true",
                    help="graph-replayed step with device timestamp marks (multi-rank capable)")
    ap.add_argument("--json-out", default=None, help="also write the table as JSON here (rank 0)")
    ap.add_argument("--ep-loopback", action="store_true",
                    help="run the fused expert-parallel kernels at world size 1 (under torchrun --nproc-per-node 1)")
    ap.add_argument("--tp", action="store_true",
                    help="N > 1: the tensor-parallel decode layout (every rank runs the same tokens; use with "
                         "--decode-only --concurrency 1 for the C=1 step)")
    a = ap.parse_args()
    import os

    import torch.distributed as dist

    from ..parallel.ep import EPGroup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    ep = tp = None
    if world > 1 or a.ep_loopback:
        # --ep-loopback: the fused expert-parallel path at world size 1 (this GPU is its only peer);
        # runs without torchrun too (one process, a one-rank group at 127.0.0.1)
        for k_, v_ in (("MASTER_ADDR", "127.0.0.1"), ("MASTER_PORT", "29599"), ("RANK", "0"), ("WORLD_SIZE", "1")):
            os.environ.setdefault(k_, v_)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        if a.tp:
            from ..parallel.tp import TPGroup
            tp = TPGroup(rank, world, dist.group.WORLD, torch.device("cuda", local), moe="ep")
        else:
            ep = EPGroup(rank, world, dist.group.WORLD, torch.device("cuda", local),
                         transport="fused" if a.ep_loopback else a.ep_transport)
    per_rank = 1 if tp is not None else world     # the tensor-parallel layout replicates the tokens
    kw = {"n_layers": a.layers} if a.layers else {}
    if a.experts:
        kw["n_routed_experts"] = a.experts
    if a.topk:
        kw["n_activated_experts"] = a.topk
    if a.family == "v41":
        from ..config import v41_flash_config
        cfg = v41_flash_config(engram_num_embeddings=(a.engram_rows, a.engram_rows), n_mtp_layers=0, **kw)
    else:
        cfg = v4_flash_config(**kw)
    dev = torch.device("cuda", local)
    n_dec = a.concurrency // per_rank - (0 if a.decode_only else 1)
    chunk = 0 if a.decode_only else a.chunk // per_rank
    T = n_dec + chunk
    max_seq = a.context + 1024 + 16
    n_phys = plan_expert_storage(cfg, dev, T, n_dec + 2, max_seq, world)
    eng = Engine.build(cfg, dev, max_seqs=n_dec + 2, max_batched_tokens=T, max_seq_len=max_seq,
                       expert_storage_layers=n_phys, use_graphs=False, ep=ep, tp=tp)
    m = eng.model
    rng = np.random.default_rng(0)     # the same seed on every rank: identical steps under --tp
    dec = a.context + (np.arange(n_dec) * (1024 // max(1, n_dec)) + 1) % 1024

    def meta(i):
        ch = [SeqChunk(s, int(dec[s]) + i, [int(rng.integers(0, cfg.vocab_size))], True) for s in range(n_dec)]
        if chunk:
            # the trace replays one graph: every step has the same shape (the chunk samples)
            samp = True if a.device_trace else i % 2 == 1
            ch.append(SeqChunk(n_dec, (i % 2) * chunk, rng.integers(0, cfg.vocab_size, chunk).tolist(), samp))
        return StepMeta(cfg, ch)

    if a.device_trace:
        _device_trace(a, eng, cfg, meta, rank, world, T, n_phys)
        return
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
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def _device_trace(a, eng, cfg, meta, rank, world, T, n_phys) -> None:
    import torch.distributed as dist

    from ..utils.devtrace import DeviceTrace, summarize

    m = eng.model
    dev = m.dev
    st = torch.cuda.Stream(dev)
    tr = DeviceTrace(dev)

    def barrier():
        if dist.is_initialized():
            dist.barrier()

    with torch.cuda.stream(st):
        # eager step with marks (fixes the mark names), then two captures: traced and plain
        m.dev_trace = tr
        mm = meta(0)
        m.upload(mm)
        tr.begin()
        m.forward(mm)
        st.synchronize()
        eng.check_errors()
        tr.freeze()
        g_tr = torch.cuda.CUDAGraph()
        mm = meta(1)
        m.upload(mm)
        with torch.cuda.graph(g_tr, stream=st):
            tr.begin()
            m.forward(mm)
        m.dev_trace = None
        g_plain = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_plain, stream=st):
            m.forward(mm)
        m.dev_trace = tr
        # warm-up replays of both graphs
        for i in range(3):
            mm = meta(2 + i)
            m.upload(mm)
            g_plain.replay()
            g_tr.replay()
        st.synchronize()
        eng.check_errors()
        # untraced step time (events around K replays)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        metas = [meta(10 + i) for i in range(a.steps)]
        e0.record(st)
        for mm in metas:
            m.upload(mm)
            g_plain.replay()
        e1.record(st)
        st.synchronize()
        plain_ms = e0.elapsed_time(e1) / a.steps
        runs, totals = [], []
        barrier()
        for i in range(a.steps):
            mm = meta(100 + i)
            m.upload(mm)
            tr.cursor = 0
            g_tr.replay()
            st.synchronize()
            tr.cursor = len(tr.names)
            runs.append(tr.read())
            totals.append(tr.total_ns() / 1e6)
        eng.check_errors()
    summ = summarize(runs)
    names = sorted(summ)
    vals = torch.tensor([summ[k]["ms"] for k in names] + [plain_ms, sum(totals) / len(totals)], dtype=torch.float64,
                        device=dev)
    vmax = vals.clone()
    if dist.is_initialized():
        dist.all_reduce(vmax, op=dist.ReduceOp.MAX)
    vmax = vmax.tolist()
    v0 = vals.tolist()
    plain_max, traced_max = vmax[-2], vmax[-1]
    if rank == 0:
        rows = sorted(((k, vmax[i], v0[i], summ[k]["n"]) for i, k in enumerate(names)), key=lambda x: -x[1])
        print(f"{'op group':20s} {'max-rank ms':>11s} {'rank0 ms':>9s} {'share':>6s}  launches-groups/step")
        for k, vx, v, n in rows:
            print(f"{k:20s} {vx:11.3f} {v:9.3f} {100 * vx / traced_max:5.1f}%  {n}")
        res = {"step_ms_graph_plain_max_rank": round(plain_max, 3), "step_ms_traced_max_rank": round(traced_max, 3),
               "T_per_rank": T, "n_layers": cfg.n_layers, "expert_storage_layers": n_phys, "world": world,
               "ops": {k: {"max_rank_ms": round(vx, 4), "rank0_ms": round(v, 4), "groups_per_step": n}
                       for k, vx, v, n in rows}}
        print(json.dumps({k: v for k, v in res.items() if k != "ops"}))
        if a.json_out:
            with open(a.json_out, "w") as f:
                json.dump(res, f, indent=1)
    del g_tr, g_plain
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
