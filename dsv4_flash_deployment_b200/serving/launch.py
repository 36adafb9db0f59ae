"""Builds the engine from an :class:`..engine.config.EngineConfig` and serves it.

Rank 0 runs the HTTP server and the engine thread; other ranks follow the
control plane (:func:`..engine.dist_engine.worker_loop`).
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

from ..engine.config import EngineConfig


def build_local_engine(ec: EngineConfig, ep=None, extra_slots: int = 0, tp=None):
    from ..engine.engine import Engine

    cfg = ec.model_config()
    if ec.device == "cpu":
        from ..io.checkpoint_spec import make_random_weights
        from ..models.oracle_step import OracleStepModel

        w = _load_weights(ec, cfg) or make_random_weights(cfg, seed=ec.seed, include_mtp=False)
        model = OracleStepModel(cfg, w, n_slots=ec.max_seqs + extra_slots, max_seq_len=ec.max_model_len)
        return Engine(model, ec.max_seqs, ec.max_batched_tokens, ec.max_model_len, ec.chunk_size, use_graphs=False)
    weights = _load_weights(ec, cfg)
    storage = ec.expert_storage_layers
    if storage is None and weights is None:
        # random init: as many distinct expert blocks as fit next to the caches and
        # step buffers (layers share blocks round-robin beyond that)
        from ..engine.memory import plan_expert_storage

        world = ep.world if ep is not None else (tp.world if tp is not None and tp.moe == "ep" else 1)
        storage = plan_expert_storage(cfg, torch.device(ec.device, torch.cuda.current_device()),
                                      ec.max_batched_tokens, ec.max_seqs + extra_slots + 1, ec.max_model_len, world)
    pool = ec.kv_pool_tokens
    if ec.kv_block and not pool and ec.gpu_memory_utilization:
        # the paged pools take what the utilization leaves after the weights and buffers
        from ..engine.memory import kv_pool_tokens_for

        dev = torch.device(ec.device, torch.cuda.current_device())
        world = ep.world if ep is not None else (tp.world if tp is not None and tp.moe == "ep" else 1)
        pool = kv_pool_tokens_for(cfg, torch.cuda.get_device_properties(dev).total_memory,
                                  ec.gpu_memory_utilization, ec.max_batched_tokens, ec.max_seqs + extra_slots + 1,
                                  ec.max_model_len, ec.kv_block, world,
                                  expert_layers=None if weights is not None else storage)
    return Engine.build(cfg, device=ec.device, max_seqs=ec.max_seqs, max_batched_tokens=ec.max_batched_tokens,
                        max_seq_len=ec.max_model_len, weights=weights, seed=ec.seed,
                        expert_storage_layers=storage, ep=ep, use_graphs=ec.use_cuda_graphs,
                        chunk_size=ec.chunk_size, extra_slots=extra_slots, tp=tp, kv_block=ec.kv_block,
                        kv_pool_tokens=pool, kv_preempt=ec.kv_preempt, engram_shm=ec.engram_shm,
                        engram_token_map=_engram_token_map(ec, cfg))


def build_spec_engine(ec: EngineConfig, local):
    """DSpark speculative decoding over the local engine's model: the MTP stages
    from the checkpoint (or drawn at random), one drafter row per cache slot."""
    from ..spec.dspark import SpecEngine
    from ..spec.serving import SpecServingEngine

    cfg = local.cfg
    if cfg.n_mtp_layers < 1:
        raise SystemExit(f"--dspark: model {cfg.name} has no MTP stages")
    spec = SpecEngine(local.model, _load_weights(ec, cfg), max_seqs=ec.max_seqs,
                      force_accept=ec.dspark_force_accept)
    return SpecServingEngine(spec, ec.max_model_len, eos_id=local.eos_id)


def _engram_token_map(ec: EngineConfig, cfg):
    """Engram hashes key on the tokenizer's normalized token texts when the served
    tokenizer has a ``tokenizer.json`` (the checkpoint's tables were built that way)."""
    if not cfg.engram_layer_ids or not ec.tokenizer:
        return None
    from pathlib import Path

    p = Path(ec.tokenizer)
    if p.is_dir():
        p = p / "tokenizer.json"
    if not p.exists():
        return None
    from ..ref.engram import compressed_token_map

    table, _ = compressed_token_map(str(p))
    if len(table) < cfg.vocab_size:   # ids the tokenizer never produces keep a map entry
        import numpy as np
        table = np.concatenate([table, np.arange(len(table), cfg.vocab_size, dtype=np.int64) % (table.max() + 1)])
    return table[:cfg.vocab_size]


def _load_weights(ec: EngineConfig, cfg):
    if ec.checkpoint is None:
        return None
    from ..io.safetensors import load_checkpoint
    return load_checkpoint(ec.checkpoint, cfg)


def init_distributed(ec: EngineConfig):
    """(rank, world, par, cpu_group) from torchrun's environment; world 1 without it.
    ``par`` is the expert-parallel group (``parallel="ep"``) or the tensor-parallel
    group (``parallel="tp"``)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        return 0, 1, None, None
    rank = int(os.environ["RANK"])
    if ec.device == "cpu":
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
        return rank, world, None, dist.group.WORLD
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=300))
    cpu_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=300))
    if ec.parallel == "tp":
        from ..parallel.tp import TPGroup
        tp = TPGroup(rank, world, dist.group.WORLD, torch.device("cuda", local), moe=ec.moe_split)
        return rank, world, tp, cpu_group
    from ..parallel.ep import EPGroup
    ep = EPGroup(rank, world, dist.group.WORLD, torch.device("cuda", local), transport=ec.ep_transport)
    return rank, world, ep, cpu_group


def main(argv: list[str] | None = None) -> None:
    from aiohttp import web

    from ..engine.dist_engine import DistributedEngine, worker_loop
    from .app import ServerState, build_app
    from .engine_loop import EngineLoop
    from .tokenizer import load_tokenizer

    ec = EngineConfig.from_args(argv)
    if ec.dspark and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--dspark serves on one GPU (the drafter runs on a whole backbone)")
    if ec.dspark and ec.device != "cuda":
        raise SystemExit("--dspark needs a CUDA device")
    rank, world, par, cpu_group = init_distributed(ec)
    if ec.device == "cuda" and world == 1:
        torch.cuda.set_device(0)
    replicated = world > 1 and ec.parallel == "tp"
    local = build_local_engine(ec, None if replicated else par, extra_slots=1 if world > 1 else 0,
                               tp=par if replicated else None)
    ctl = None
    if world > 1:
        from ..engine.control import make_control
        ctl = make_control(ec.control_plane, cpu_group)
    if rank != 0:
        worker_loop(local, cpu_group, replicated=replicated, control=ctl)
        local.graphs.clear()
        dist.destroy_process_group()
        return
    eng = DistributedEngine(local, cpu_group, replicated=replicated, control=ctl) if world > 1 else local
    if ec.dspark:
        eng = build_spec_engine(ec, local)
    loop = EngineLoop(eng, step_deadline_s=ec.step_deadline_s).start()
    tok = load_tokenizer(ec.tokenizer, local.cfg)
    info = {"device": ec.device, "world_size": world, "engine_config": ec.to_dict()}
    if ec.device == "cuda":
        info["device_name"] = torch.cuda.get_device_name()
    st = ServerState(loop, tok, ec.served_model_name, ec.max_model_len, info,
                     api_key=ec.api_key or os.environ.get("DSV4_API_KEY") or None)
    try:
        app = build_app(st)

        async def drain(_app):
            # SIGTERM / SIGINT: /health answers 503 "draining", new requests are refused,
            # live ones run to completion for up to drain_timeout_s
            import asyncio
            await asyncio.to_thread(loop.drain, ec.drain_timeout_s)
        app.on_shutdown.append(drain)
        web.run_app(app, host=ec.host, port=ec.port, print=None, shutdown_timeout=ec.drain_timeout_s + 5)
    finally:
        loop.stop()
        if world > 1:
            eng.shutdown()
            dist.destroy_process_group()
