"""HBM budgeting for a model instance on one GPU (180 GB B200).

Estimates everything that is not routed-expert weight (dense weights, the
caches, step buffers, runtime reserve) and returns how many distinct physical
expert blocks fit.  When fewer blocks than layers fit, layers share blocks
round-robin (random-init benchmark runs only); each layer still streams a full
block from HBM, so the work per step is unchanged.
"""

from __future__ import annotations

import torch

from ..models.kv_format import ik4_bytes, kv4_bytes, kv8_bytes


def expert_block_bytes(cfg, ep_world: int = 1) -> int:
    e_local = cfg.n_routed_experts // ep_world
    per = 3 * cfg.dim * cfg.moe_inter_dim
    if cfg.expert_format == "mxfp4":
        return int(e_local * per * (0.5 + 1 / 32))
    return int(e_local * per * (1 + 1 / 32))


def non_expert_bytes(cfg, max_tokens: int, n_slots: int, max_seq: int, kv_block: int = 0,
                     kv_pool_tokens: int = 0) -> int:
    """``kv_block`` > 0: the compressed caches are paged pools of ``kv_pool_tokens``
    tokens of context (0: ``n_slots * max_seq``) plus one scratch block per ratio."""
    d = cfg.dim
    per_layer = ((cfg.q_lora_rank + cfg.head_dim) * d + cfg.q_dim * cfg.q_lora_rank + 2 * cfg.o_inter * cfg.o_group_in
                 + d * cfg.o_inter + 3 * d * cfg.n_shared_experts * cfg.moe_inter_dim
                 + 2 * cfg.n_routed_experts * d + 2 * 2 * cfg.hc_rows * cfg.hc_mult * d * 2)
    dense = cfg.n_layers * per_layer
    for l in cfg.kv_source_layer_ids:
        dense += 2 * 2 * cfg.overlap(l) * cfg.head_dim * d
    for l in cfg.index_source_layer_ids:
        dense += cfg.index_n_heads * cfg.index_head_dim * cfg.q_lora_rank + 2 * 128 * d
    emb = 2 * 2 * cfg.vocab_size * d
    s = n_slots + 1
    # window rows are KV8 records, compressed rows KV4, indexer keys IK4 (models/kv_format.py)
    kv = cfg.n_layers * s * cfg.sliding_window * kv8_bytes(cfg.head_dim)
    for l in cfg.kv_source_layer_ids:
        r, co = cfg.ratio(l), cfg.overlap(l)
        if kv_block:
            pool = kv_pool_tokens or n_slots * max_seq
            rows = (-(-max(1, pool // r) // kv_block) + 1) * kv_block
        else:
            rows = s * (max_seq // r)
        kv += rows * kv4_bytes(cfg.head_dim) + s * co * r * 2 * co * cfg.head_dim * 4
        if l in cfg.index_source_layer_ids:
            kv += rows * ik4_bytes(cfg.index_head_dim)
    t = max_tokens
    k = cfg.n_activated_experts
    cap = t * k * 2 + cfg.n_routed_experts * 128
    step = (t * (cfg.hc_mult * d * 2 + 6 * d + 2 * 2 * cfg.q_dim + 6 * cfg.o_inter + 16 * cfg.head_dim)
            + cap * (d * 3 + cfg.moe_inter_dim * 2) + t * cfg.vocab_size * 4 + 64 * 2 ** 20)
    return dense + emb + kv + step


def plan_expert_storage(cfg, device, max_tokens: int, n_slots: int, max_seq: int, ep_world: int = 1,
                        reserve_gb: float = 10.0) -> int:
    free, _ = torch.cuda.mem_get_info(device)
    avail = free - non_expert_bytes(cfg, max_tokens, n_slots, max_seq) - int(reserve_gb * 2 ** 30)
    n = int(avail // expert_block_bytes(cfg, ep_world))
    return max(1, min(cfg.n_layers, n))


def kv_pool_tokens_for(cfg, total_bytes: int, utilization: float, max_tokens: int, n_slots: int, max_seq: int,
                       kv_block: int, ep_world: int = 1, expert_layers: int | None = None) -> int:
    """Tokens of context the paged compressed-cache pools can hold when the instance
    may use ``utilization`` of ``total_bytes`` of HBM (vLLM's
    ``--gpu-memory-utilization``, which the reference serves with at 0.85): the
    budget minus the expert blocks of ``expert_layers`` layers (all layers by
    default, as with a checkpoint) and everything else that is not pool, divided
    by the pool's bytes per token of context.  Rounded down to whole blocks of
    the largest ratio; at least one request of ``max_seq`` tokens must fit."""
    if not 0.0 < utilization <= 1.0:
        raise ValueError("gpu memory utilization must be in (0, 1]")
    layers = cfg.n_layers if expert_layers is None else expert_layers
    experts = layers * expert_block_bytes(cfg, ep_world)
    p0, p1 = max_seq, max_seq + (1 << 20)
    b0 = non_expert_bytes(cfg, max_tokens, n_slots, max_seq, kv_block, p0)
    b1 = non_expert_bytes(cfg, max_tokens, n_slots, max_seq, kv_block, p1)
    per_token = (b1 - b0) / (p1 - p0)
    spare = utilization * total_bytes - experts - b0
    pool = p0 + int(spare // per_token) if per_token > 0 else p0
    step = max(cfg.ratio(l) for l in cfg.kv_source_layer_ids) * kv_block
    pool = pool // step * step
    if pool < max_seq:
        raise ValueError(f"{utilization:.2f} of {total_bytes / 2 ** 30:.1f} GiB holds the weights and buffers but "
                         f"not one {max_seq}-token request's caches")
    return pool
