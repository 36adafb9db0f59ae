"""Checkpoint tensor inventory and deterministic random-init weights.

The tensor names, dtypes and shapes are the reference checkpoint layout
(``models/DeepSeekV4.1-Flash-v6e16/tpu-v7x/deepseek_v41/checkpoint.py:73-202``):
dense projections are FP8 e4m3 with 32x32-block ue8m0 scales, routed experts
are packed e2m1 pairs (``I8``) with per-32 ue8m0 scales, compressor/indexer
projections are BF16 and mHC parameters F32.  V4-Flash-shaped configs add the
compressor position embedding (``attn.compressor.ape``) and store experts as
MXFP8 (e4m3 with per-32 ue8m0 scales), which the benchmark definition asks for.

Random init: every tensor is drawn from a generator seeded by (seed, name), so
any subset of tensors (one rank's shard, one layer) can be produced alone and
matches the same tensor produced as part of the whole.
"""

from __future__ import annotations

import hashlib
from typing import Iterable

import torch

# dtype tags (safetensors names)
F8 = "F8_E4M3"
E8 = "F8_E8M0"
I8 = "I8"
BF16 = "BF16"
F32 = "F32"

TORCH_DTYPE = {
    F8: torch.float8_e4m3fn,
    E8: torch.uint8,
    I8: torch.int8,
    BF16: torch.bfloat16,
    F32: torch.float32,
}


def _layer_specs(cfg, prefix: str, layer_id: int, backbone: bool) -> dict[str, tuple[str, tuple[int, ...]]]:
    s: dict[str, tuple[str, tuple[int, ...]]] = {}
    d = cfg.dim
    s[f"{prefix}.attn.attn_sink"] = (F32, (cfg.n_heads,))
    s[f"{prefix}.attn.kv_norm.weight"] = (BF16, (cfg.head_dim,))
    s[f"{prefix}.attn.q_norm.weight"] = (BF16, (cfg.q_lora_rank,))

    def fp8(name: str, n: int, k: int) -> None:
        s[f"{prefix}.{name}.weight"] = (F8, (n, k))
        s[f"{prefix}.{name}.scale"] = (E8, (n // 32, k // 32))

    fp8("attn.wq_a", cfg.q_lora_rank, d)
    fp8("attn.wq_b", cfg.q_dim, cfg.q_lora_rank)
    fp8("attn.wkv", cfg.head_dim, d)
    fp8("attn.wo_a", cfg.o_inter, cfg.o_group_in)
    fp8("attn.wo_b", d, cfg.o_inter)

    if backbone and layer_id in cfg.kv_source_layer_ids:
        r = cfg.ratio(layer_id)
        width = cfg.overlap(layer_id) * cfg.head_dim
        s[f"{prefix}.attn.compressor.norm.weight"] = (BF16, (cfg.head_dim,))
        s[f"{prefix}.attn.compressor.wkv.weight"] = (BF16, (width, d))
        if r > 1:
            s[f"{prefix}.attn.compressor.wgate.weight"] = (BF16, (width, d))
            if cfg.compressor_ape:
                s[f"{prefix}.attn.compressor.ape"] = (F32, (r, width))
    if backbone and layer_id in cfg.index_source_layer_ids:
        if layer_id in cfg.kv_source_layer_ids:
            s[f"{prefix}.attn.indexer.k_norm.weight"] = (BF16, (cfg.index_head_dim,))
            s[f"{prefix}.attn.indexer.wk.weight"] = (BF16, (cfg.index_head_dim, cfg.head_dim))
        s[f"{prefix}.attn.indexer.weights_proj.weight"] = (BF16, (cfg.index_n_heads, d))
        fp8("attn.indexer.wq_b", cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank)

    s[f"{prefix}.attn_norm.weight"] = (BF16, (d,))
    s[f"{prefix}.ffn_norm.weight"] = (BF16, (d,))
    for which in ("attn", "ffn"):
        s[f"{prefix}.hc_{which}_base"] = (F32, (cfg.hc_rows,))
        s[f"{prefix}.hc_{which}_fn"] = (F32, (cfg.hc_rows, cfg.hc_mult * d))
        s[f"{prefix}.hc_{which}_scale"] = (F32, (3,))

    n_exp = cfg.n_experts_for(layer_id)
    inter = cfg.moe_inter_dim
    for e in range(n_exp):
        ep = f"{prefix}.ffn.experts.{e}"
        if cfg.expert_format == "mxfp4":
            s[f"{ep}.w1.weight"] = (I8, (inter, d // 2))
            s[f"{ep}.w3.weight"] = (I8, (inter, d // 2))
            s[f"{ep}.w2.weight"] = (I8, (d, inter // 2))
        else:
            s[f"{ep}.w1.weight"] = (F8, (inter, d))
            s[f"{ep}.w3.weight"] = (F8, (inter, d))
            s[f"{ep}.w2.weight"] = (F8, (d, inter))
        s[f"{ep}.w1.scale"] = (E8, (inter, d // 32))
        s[f"{ep}.w3.scale"] = (E8, (inter, d // 32))
        s[f"{ep}.w2.scale"] = (E8, (d, inter // 32))
    s[f"{prefix}.ffn.gate.bias"] = (F32, (n_exp,))
    if cfg.family == "v4.1":
        # the V4.1 checkpoint's second routing bias, for image-sentinel tokens; text
        # tokens route with ``gate.bias``, so this text-only engine loads it and never
        # reads it (the reference's tensor list holds it: checkpoint.py:145)
        s[f"{prefix}.ffn.gate.bias_vl"] = (F32, (n_exp,))
    s[f"{prefix}.ffn.gate.weight"] = (BF16, (n_exp, d))
    si = cfg.n_shared_experts * inter
    fp8("ffn.shared_experts.w1", si, d)
    fp8("ffn.shared_experts.w3", si, d)
    fp8("ffn.shared_experts.w2", d, si)

    if backbone and layer_id in cfg.engram_layer_ids:
        i = cfg.engram_layer_ids.index(layer_id)
        n_emb = cfg.engram_num_embeddings[i]
        e_in = (cfg.engram_max_ngram_size - 1) * cfg.engram_n_heads * cfg.engram_head_dim
        s[f"{prefix}.engram.embed.weight"] = (F8, (n_emb, cfg.engram_head_dim))
        s[f"{prefix}.engram.embed.scale"] = (E8, (n_emb, cfg.engram_head_dim // 32))
        s[f"{prefix}.engram.k_weight"] = (BF16, (cfg.hc_mult, d))
        s[f"{prefix}.engram.q_weight"] = (BF16, (cfg.hc_mult, d))
        fp8("engram.wkv", (cfg.hc_mult + 1) * d, e_in)
    return s


def checkpoint_specs(cfg, include_mtp: bool = True) -> dict[str, tuple[str, tuple[int, ...]]]:
    """``{name: (dtype_tag, shape)}`` for the whole model."""
    s: dict[str, tuple[str, tuple[int, ...]]] = {"embed.weight": (BF16, (cfg.vocab_size, cfg.dim))}
    for lid in range(cfg.n_layers):
        s.update(_layer_specs(cfg, f"layers.{lid}", lid, True))
    s["head.weight"] = (BF16, (cfg.vocab_size, cfg.dim))
    s["norm.weight"] = (BF16, (cfg.dim,))
    if include_mtp:
        for k in range(cfg.n_mtp_layers):
            p = f"mtp.{k}"
            s.update(_layer_specs(cfg, p, cfg.n_layers + k, False))
            if k == 0:
                s[f"{p}.main_norm.weight"] = (BF16, (cfg.dim,))
                s[f"{p}.main_proj.weight"] = (F8, (cfg.dim, len(cfg.dspark_target_layer_ids) * cfg.dim))
                s[f"{p}.main_proj.scale"] = (E8, (cfg.dim // 32, len(cfg.dspark_target_layer_ids) * cfg.dim // 32))
            if k == cfg.n_mtp_layers - 1:
                s[f"{p}.confidence_head.proj.weight"] = (BF16, (1, cfg.dim + cfg.markov_rank))
                s[f"{p}.markov_head.embed.weight"] = (BF16, (cfg.vocab_size, cfg.markov_rank))
                s[f"{p}.markov_head.head.weight"] = (BF16, (cfg.vocab_size, cfg.markov_rank))
                s[f"{p}.norm.weight"] = (BF16, (cfg.dim,))
    return s


def _seed_for(seed: int, name: str) -> int:
    h = hashlib.blake2b(f"{seed}:{name}".encode(), digest_size=8).digest()
    return int.from_bytes(h, "little") & 0x7FFF_FFFF_FFFF_FFFF


def random_tensor(name: str, tag: str, shape: tuple[int, ...], seed: int = 0,
                  device: str | torch.device = "cpu", mxfp4_experts: bool = False,
                  init_std: float | None = None) -> torch.Tensor:
    """One deterministic random tensor for checkpoint entry ``name``.

    Default: scales are powers of two near 2^-7 so block-scaled weights have
    unit-ish gain per sqrt(fan-in); BF16 matrices are N(0, 1/fan_in); norm
    weights ~1.  With ``init_std`` every weight matrix dequantizes to
    ~N(0, init_std) (FP8 codes ~N(0, init_std * 32) under a 2^-5 scale), norm
    weights are 1 and mHC parameters keep their defaults.
    """
    g = torch.Generator(device=device)
    g.manual_seed(_seed_for(seed, name))
    dev = torch.device(device)
    if init_std is not None and tag in (E8, F8, BF16):
        if tag == E8:
            return torch.full(shape, 122, dtype=torch.uint8, device=dev)
        if tag == F8:
            v = (torch.randn(shape, generator=g, device=dev) * (init_std * 32.0)).to(torch.float8_e4m3fn)
            v.view(torch.uint8)[v.view(torch.uint8) == 0x80] = 0
            return v
        if name.endswith("norm.weight"):
            return torch.ones(shape, dtype=torch.bfloat16, device=dev)
        return (torch.randn(shape, generator=g, device=dev) * init_std).to(torch.bfloat16)
    if tag == E8:
        # MXFP4 expert codes span +-6 (vs ~N(0, 0.5) for e4m3 values): their scales sit
        # 3 binades lower so both expert formats have the same weight magnitude.
        lo = 115 if (".experts." in name and name.endswith(".scale") and mxfp4_experts) else 118
        return torch.randint(lo, lo + 5, shape, generator=g, device=dev, dtype=torch.int32).to(torch.uint8)
    if tag == I8:
        return torch.randint(-128, 128, shape, generator=g, device=dev, dtype=torch.int32).to(torch.int8)
    if tag == F8:
        v = (torch.randn(shape, generator=g, device=dev) * 0.5).to(torch.float8_e4m3fn)
        u = v.view(torch.uint8)
        u[u == 0x80] = 0  # no negative zero, as in the reference generator
        return v
    if tag == BF16:
        if name.endswith("norm.weight"):
            v = 1.0 + 0.05 * torch.randn(shape, generator=g, device=dev)
        else:
            fan_in = shape[-1] if len(shape) >= 2 else shape[0]
            v = torch.randn(shape, generator=g, device=dev) / (fan_in ** 0.5)
        return v.to(torch.bfloat16)
    if tag == F32:
        v = torch.randn(shape, generator=g, device=dev)
        if name.endswith("_scale"):
            return torch.full(shape, 0.25, device=dev)
        if name.endswith("_base"):
            return v * 0.05
        if name.endswith("_fn"):
            return v * 0.02
        if name.endswith("attn_sink"):
            return v * 0.1 - 2.0
        return v * 0.02
    raise ValueError(f"unhandled dtype tag {tag} for {name}")


def make_random_weights(cfg, seed: int = 0, device: str | torch.device = "cpu",
                        names: Iterable[str] | None = None, include_mtp: bool = True,
                        init_std: float | None = None) -> dict[str, torch.Tensor]:
    specs = checkpoint_specs(cfg, include_mtp=include_mtp)
    keys = list(specs) if names is None else list(names)
    mx4 = cfg.expert_format == "mxfp4"
    return {k: random_tensor(k, specs[k][0], specs[k][1], seed, device, mx4, init_std) for k in keys}
