"""DeepSeek-V4.1-Flash benchmark on the full-size model (random init, one GPU or EP over N).

Measures, for the V4.1 architecture (552B: 40 layers + 3 DSpark stages, 384
MXFP4 experts top-6, ratio-2/ratio-1 compressed attention + SWA, 4-stream mHC,
Engram at layers 1 and 14 with its tables in page-locked host memory):

* output tok/s of the 1k/1k steady-state step at concurrency C (default 190,
  the hybrid fused-MoE row of the reference, ``FK/results/raw/1k1k-c190.json``):
  C-1 decoding sequences + one prefill chunk per step, CUDA-graph replay,
  device-timed (max over ranks);
* C=1 TPOT: one sequence, 1-token steps through ``Engine.run_meta`` (pinned
  H2D + D2H + host sync every token), graph replay (reference megakernel
  9.18 ms, ``MK/results/megakernel_v6e16_results.json:685``); on N > 1 GPUs
  on the tensor-parallel layout (heads, ``wo_a`` groups, ``wo_b`` columns and
  head rows split over the ranks, the batch model's expert blocks and Engram
  runtime shared), with the batch layout's value beside it;
* C=1 effective TPOT with DSpark 1+4 (single GPU): draft (3 MTP stages +
  Markov chain) + verify (5 tokens through the target) + ring commit + ingest
  per round, with the reference's forced-acceptance knob (random weights
  accept nothing by themselves, ``deepseek_v41/engine.py:332``); effective
  TPOT = round wall time / emitted tokens (reference 7.27 ms, ``:784``).

Engram tables: the reference's two tables are ~101 GB each; the GPU hosts of
this pool have 196 GB of RAM, so ``--engram-rows`` sizes them (default 2 x 96M
rows = 2 x 25 GB page-locked); hashing and the per-token row reads (24 rows x
264 bytes per token and layer) are the same at any table size.

    python -m dsv4_flash_deployment_b200.bench.v41_bench --steps 6 --warmup 3
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import time

import numpy as np
import torch
import torch.distributed as dist

FK_C190 = 1471.6       # tok/s, FK/results/raw/1k1k-c190.json (TPU v6e-16, raw)
MK_TPOT = 9.18         # ms, MK/results/megakernel_v6e16_results.json:685
MK_SPEC_TPOT = 7.27    # ms, MK/results/megakernel_v6e16_results.json:784


def _timed(stream, fn, n: int) -> tuple[float, float]:
    """(device ms, wall ms) per call of fn over n calls."""
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record(stream)
    for i in range(n):
        fn(i)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n, (time.perf_counter() - w0) / n * 1e3


def parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser()
    ap.add_argument("--concurrency", type=int, default=190)
    ap.add_argument("--steps", type=int, default=6)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--isl", type=int, default=1024)
    ap.add_argument("--osl", type=int, default=1024)
    ap.add_argument("--chunk", type=int, default=256, help="prefill tokens per step (the reference's V4.1 chunk)")
    ap.add_argument("--engram-rows", type=int, default=96_000_000, help="rows per Engram table")
    ap.add_argument("--engram-shm", default=None,
                    help="keep the Engram tables in shared files with this prefix (e.g. /dev/shm/dsv4_engram): "
                         "one copy per node instead of one per rank")
    ap.add_argument("--spec-rounds", type=int, default=12)
    ap.add_argument("--force-accept", default="2.15,4",
                    help="accepted drafts per round, comma list; fractional values alternate floor/ceil "
                         "(2.15 = the reference's measured 3.15 tokens per round)")
    ap.add_argument("--no-spec", action="store_true")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--no-tp", action="store_true", help="N>1: skip the tensor-parallel C=1 measurement")
    ap.add_argument("--ep-transport", default="fused", choices=["p2p", "nccl", "fused"])
    return ap


def main(argv=None) -> None:
    a = parser().parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
        group = dist.group.WORLD
    line = measure(a, dev, rank, world, group)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if group is not None:
        dist.barrier()
        dist.destroy_process_group()


def measure(a, dev, rank: int, world: int, group) -> dict:
    """Runs every V4.1 measurement on this rank (the process group, if any, is
    already up); returns the result line (complete on rank 0)."""

    from ..config import v41_flash_config
    from ..engine.engine import Engine
    from ..engine.memory import expert_block_bytes, plan_expert_storage
    from ..models.model import SeqChunk, StepMeta
    from ..parallel import ep as ep_mod
    from ..utils.provenance import provenance

    cfg = v41_flash_config(engram_num_embeddings=(a.engram_rows, a.engram_rows))
    C = a.concurrency
    c_rank = max(2, C // world)
    n_dec = c_rank - 1
    chunk = max(1, a.chunk // world)
    max_tokens = n_dec + chunk
    max_seq = a.isl + a.osl
    ep = ep_mod.EPGroup(rank, world, group, dev, transport=a.ep_transport) if world > 1 else None
    # the DSpark stages' expert blocks (3 x 128 experts) come out of the reserve
    spec_gb = 0 if a.no_spec else cfg.n_mtp_layers * expert_block_bytes(
        dataclasses.replace(cfg, n_routed_experts=cfg.dspark_n_routed_experts), 1) / 2 ** 30
    tp_gb = 8.0 if world > 1 and not a.no_tp else 0.0      # the tensor-parallel C=1 model's dense shards
    n_phys = plan_expert_storage(cfg, dev, max_tokens, c_rank + 1, max_seq, world, reserve_gb=12.0 + spec_gb + tp_gb)
    t_build = time.perf_counter()
    eng = Engine.build(cfg, dev, max_seqs=c_rank + 1, max_batched_tokens=max_tokens, max_seq_len=max_seq,
                       expert_storage_layers=n_phys, ep=ep, use_graphs=not a.no_graphs, chunk_size=chunk,
                       engram_shm=a.engram_shm)
    t_build = time.perf_counter() - t_build
    model = eng.model
    rng = np.random.default_rng(99 + rank)

    # ---------------------------------------------------- 1k/1k steady state
    dec_pos = (a.isl + (np.arange(n_dec) * (a.osl // max(1, n_dec)) + 1) % a.osl).astype(np.int64)
    state = {"pre": 0, "dec": dec_pos.copy()}

    def make_meta():
        chunks = [SeqChunk(s, int(state["dec"][s]), [int(rng.integers(0, cfg.vocab_size))], True)
                  for s in range(n_dec)]
        p0 = state["pre"]
        chunks.append(SeqChunk(n_dec, p0, rng.integers(0, cfg.vocab_size, chunk).tolist(), True))
        state["dec"] = np.where(state["dec"] + 1 >= max_seq, a.isl, state["dec"] + 1)
        state["pre"] = (p0 + chunk) % a.isl
        return StepMeta(cfg, chunks)

    for _ in range(a.warmup):
        eng.run_meta(make_meta())
    eng.check_errors()
    metas = [make_meta() for _ in range(a.steps)]
    if group is not None:
        dist.barrier()
    ms, _ = _timed(eng.stream, lambda i: eng.run_meta(metas[i]), a.steps)
    eng.check_errors()
    ms_t = torch.tensor([ms], device=dev)
    if group is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    tok_s = n_dec * world / (ms / 1e3)

    # ---------------------------------------------------------- C=1 plain
    c1_pos = a.isl + a.osl // 2
    c1 = lambda i: StepMeta(cfg, [SeqChunk(0, c1_pos + i, [int(rng.integers(0, cfg.vocab_size))], True)])
    for i in range(3):
        eng.run_meta(c1(i))
    c1m = [c1(3 + i) for i in range(max(8, a.steps))]
    if group is not None:
        dist.barrier()
    c1_dev, c1_wall = _timed(eng.stream, lambda i: eng.run_meta(c1m[i]), len(c1m))
    eng.check_errors()

    # -------------------------------------------- C=1 tensor parallel (N > 1)
    c1_tp = None
    if world > 1 and not a.no_tp:
        from ..parallel.tp import TPGroup
        tpg = TPGroup(rank, world, group, dev, moe="ep")
        eng_tp = Engine.build(cfg, dev, max_seqs=2, max_batched_tokens=16, max_seq_len=max_seq, tp=tpg,
                              experts_from=model, engram_from=model, use_graphs=not a.no_graphs, chunk_size=16)
        rng_tp = np.random.default_rng(4321)   # the same tokens on every rank
        tpm = [StepMeta(cfg, [SeqChunk(0, c1_pos + i, [int(rng_tp.integers(0, cfg.vocab_size))], True)])
               for i in range(3 + len(c1m))]
        for i in range(3):
            eng_tp.run_meta(tpm[i])
        eng_tp.check_errors()
        dist.barrier()
        tp_dev, tp_wall = _timed(eng_tp.stream, lambda i: eng_tp.run_meta(tpm[3 + i]), len(c1m))
        eng_tp.check_errors()
        tp_t = torch.tensor([tp_dev, tp_wall], device=dev)
        dist.all_reduce(tp_t, op=dist.ReduceOp.MAX)
        c1_tp = tuple(float(x) for x in tp_t.tolist())
        eng_tp.graphs.clear()
        del eng_tp
        tpg.release()
        dist.barrier()

    # ------------------------------------------------ C=1 DSpark 1+4 (1 GPU)
    spec = None
    if not a.no_spec and world == 1:
        from ..spec.dspark import SpecEngine
        eng.graphs.clear()
        accepts = [float(x) for x in str(a.force_accept).split(",") if x]
        se = SpecEngine(model, None, max_seqs=1, force_accept=accepts[0])
        prompt = rng.integers(0, cfg.vocab_size, a.isl).tolist()
        se.prefill([prompt])

        def round_(_i):
            toks = se.draft([0])
            blocks = [[se.outs[0][-1]] + [int(toks[i + 1, 0]) for i in range(se.blk - 1)]]
            se.verify([0], blocks)

        from ..ops.gemm import ErrorWord
        runs = []
        for f in accepts:
            se.force_accept, se._forced_rounds = f, 0
            for i in range(2):
                round_(i)
            se._forced_rounds = 0
            e0 = se.stats.emitted
            r_dev, r_wall = _timed(torch.cuda.current_stream(dev), round_, a.spec_rounds)
            emitted = (se.stats.emitted - e0) / a.spec_rounds
            ErrorWord.check(dev)
            runs.append({"effective_tpot_ms": round(r_wall / emitted, 3), "round_ms": round(r_wall, 3),
                         "round_device_ms": round(r_dev, 3), "tokens_per_round": round(emitted, 3),
                         "force_accept": f})
        spec = dict(runs[0])
        spec.update({"by_acceptance": runs, "baseline_ms": MK_SPEC_TPOT,
                     "baseline_tokens_per_round": 3.15,
                     "note": "eager rounds: draft (3 MTP stages + Markov chain, host reads the block) + verify "
                             "(5 tokens, deferred rings) + ring commit + main-hidden ingest; prompt of isl tokens; "
                             "the first entry forces the reference's measured mean acceptance"})

    line = {}
    if rank == 0:
        eg = model.engram
        tables_gb = sum(t.q.numel() + t.sf.numel() for t in eg.tables) / 2 ** 30 if eg is not None else 0
        line = {
            "metric": f"V4.1-Flash output tok/s @1k/1k C={C} (max over ranks); C=1 TPOT; DSpark effective TPOT",
            "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": round(tok_s / FK_C190, 3), "dtype": "bf16",
            "data": "synthetic: uniform-random token ids, random-init weights",
            "config": {"model": "deepseek-v4.1-flash (40L + 3 MTP, d5120, 384 experts top-6 inter2304 MXFP4, "
                                "Engram L1/L14)",
                       "global_batch": C, "seq_len": max_seq,
                       "workload": f"1k1k C={C} steady-state step: {n_dec * world} decode + {chunk * world} "
                                   "prefill tokens",
                       "parallelism": f"dp-attention{world} x ep{world}" if world > 1 else "single GPU",
                       "expert_storage_layers": n_phys, "cuda_graphs": not a.no_graphs,
                       "l2": "inputs larger than L2 (experts 7.2 GB per layer)",
                       "engram": {"rows_per_table": a.engram_rows, "tables_gb_pinned_host": round(tables_gb, 1),
                                  "shared_files": a.engram_shm,
                                  "note": "reference tables 2 x ~101 GB exceed the 196 GB host RAM of the GPU box"},
                       "build_s": round(t_build, 1)},
            "c1_tpot_ms": ({"value": round(c1_wall, 3), "device_ms": round(c1_dev, 3), "context": c1_pos,
                            "layout": "single GPU", "baseline_ms": MK_TPOT} if c1_tp is None else
                           {"value": round(c1_tp[1], 3), "device_ms": round(c1_tp[0], 3), "context": c1_pos,
                            "layout": f"tp{world} attention + ep{world} experts, Engram whole on every rank",
                            "batch_layout_ms": round(c1_wall, 3), "baseline_ms": MK_TPOT}),
            "dspark": spec,
            "hardware": provenance(dev),
        }
    eng.graphs.clear()
    if ep is not None:
        ep.release()
    return line


if __name__ == "__main__":
    main()
