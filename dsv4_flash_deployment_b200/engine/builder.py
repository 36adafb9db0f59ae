"""Model construction: checkpoint tensors or device-side random init."""

from __future__ import annotations

import torch

from ..models.model import DSV4Model
from ..models.weights import load_layer, random_experts, random_layer
from ..ops.layout import ceil_to


def _pad_rows(w: torch.Tensor) -> torch.Tensor:
    n = w.shape[0]
    npad = ceil_to(n, 128)
    if npad == n:
        return w.contiguous()
    out = torch.zeros(npad, *w.shape[1:], dtype=w.dtype, device=w.device)
    out[:n] = w
    return out


def build_model(cfg, device="cuda", max_tokens: int = 512, n_slots: int = 16, max_seq_len: int = 2048,
                weights: dict | None = None, seed: int = 0, expert_storage_layers: int | None = None,
                ep=None, tp=None, experts_from: DSV4Model | None = None, kv_block: int = 0,
                kv_pool_tokens: int = 0, engram_from: DSV4Model | None = None,
                engram_shm: str | None = None, engram_token_map=None,
                merge_shared: bool | None = None) -> DSV4Model:
    """Builds the backbone.

    ``weights``: checkpoint dict (names of the reference checkpoint); None draws
    random weights on the device.  ``expert_storage_layers``: with random init,
    the number of distinct physical expert blocks (layers share them round-robin
    when the model does not fit one GPU).  ``ep``: expert-parallel group.
    ``tp``: tensor-parallel group (parallel/tp.py): every rank draws or loads the
    full weights with the same seed and keeps its shard of heads, output groups,
    wo_b columns, experts and head rows.  ``experts_from``: random init only; the
    layers reuse that model's expert blocks (a second layout of the same model on
    the same GPUs, e.g. tensor-parallel decode next to the expert-parallel batch).
    ``kv_block``: entries per block of the paged compressed caches (0: one
    contiguous ``max_seq_len`` cache per slot); ``kv_pool_tokens``: pool size in
    tokens of context (0: ``n_slots * max_seq_len``).  ``engram_from``: a model
    whose Engram runtime (host tables, token rings, staging buffers) this one
    uses instead of building its own; it must have at least as many slots and
    step tokens, and the two models must not step concurrently.  ``engram_shm``:
    random-init Engram tables in shared files with this prefix (one copy per node).
    ``engram_token_map``: the tokenizer's compressed token map for the Engram
    hashes (``ref.engram.compressed_token_map``; None: ``id % C``).
    ``merge_shared``: the shared expert's tiles ride in the routed experts' grouped
    GEMMs where the layout allows it (None: ``DSV4_MERGE_SHARED``, default on;
    False: two separate dense GEMMs).
    """
    dev = torch.device(device)
    if tp is not None and ep is not None:
        raise ValueError("tensor parallelism owns the experts itself; pass tp or ep, not both")
    par = ep if ep is not None else tp
    e_begin, e_local = 0, cfg.n_routed_experts
    if par is not None:
        e_begin, e_local = par.expert_range(cfg.n_routed_experts)
    layers = []
    if weights is not None:
        for lid in range(cfg.n_layers):
            rng = par.expert_range(cfg.n_experts_for(lid)) if par is not None else None
            L = load_layer(cfg, weights, lid, dev, expert_range=rng)
            if tp is not None and tp.moe == "tp":
                L.experts = tp.shard_experts(L.experts)   # this rank's intermediate slice
            layers.append(L)
        embed = weights["embed.weight"].to(dev)
        head = _pad_rows(weights["head.weight"]).to(dev)
        norm = weights["norm.weight"].to(dev)
    else:
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        if experts_from is not None:
            stores = [L.experts for L in experts_from.layers]
            if stores[0].n_experts != e_local:
                raise ValueError("shared expert blocks belong to a different expert split")
        else:
            n_phys = expert_storage_layers or cfg.n_layers
            inter = tp.inter_local(cfg.moe_inter_dim) if tp is not None else None
            stores = [random_experts(cfg, e_local, dev, g, inter=inter) for _ in range(min(n_phys, cfg.n_layers))]
        for lid in range(cfg.n_layers):
            layers.append(random_layer(cfg, lid, dev, g, stores[lid % len(stores)]))
        embed = (torch.randn(cfg.vocab_size, cfg.dim, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        head = _pad_rows((torch.randn(cfg.vocab_size, cfg.dim, device=dev, generator=g) / cfg.dim ** 0.5)
                         .to(torch.bfloat16))
        norm = (1.0 + 0.05 * torch.randn(cfg.dim, device=dev, generator=g)).to(torch.bfloat16)
    if tp is not None:
        for L in layers:
            tp.shard_layer(cfg, L)
        head = tp.shard_head(head, cfg.vocab_size)
    model = DSV4Model(cfg, layers, embed, head, norm, max_tokens, n_slots, max_seq_len, dev, ep=ep,
                      head_vocab=cfg.vocab_size, tp=tp, kv_block=kv_block, kv_pool_tokens=kv_pool_tokens,
                      merge_shared=merge_shared)
    if cfg.engram_layer_ids and engram_from is not None:
        eg = engram_from.engram
        if eg is None or eg.ring.shape[0] < n_slots + 1 or eg.rows.shape[0] < max_tokens:
            raise ValueError("engram_from: runtime missing or smaller than this model's slots / step tokens")
        model.engram = eg
    elif cfg.engram_layer_ids:
        from ..models.engram import EngramRuntime
        # + 1: the padding slot (bucketed steps and idle ranks park their tokens there)
        model.engram = EngramRuntime(cfg, dev, n_slots + 1, max_tokens, model.ext, weights=weights, seed=seed,
                                     shm_prefix=engram_shm, token_map=engram_token_map)
    return model
