"""Model configuration for the DeepSeek-V4 family served by this engine.

One dataclass covers both model families the reference serves:

* DeepSeek-V4.1-Flash (552B / 16B active): every field default below is the
  V4.1 value, taken from the reference's architecture record
  (``models/DeepSeekV4.1-Flash-v6e16/tpu-v7x/deepseek_v41/config.py:24-81``;
  layer kinds ``:11-21``, kv/index source rules ``:102-129``).
* DeepSeek-V4-Flash (284B / 13B active, 256 experts top-8, CSA r=4 + HCA
  r=128). The reference never states its dimensions; it only serves the
  upstream model.  :func:`v4_flash_config` fixes the MoE shape from the
  benchmark definition (hidden 4096, 256 experts, inter 2048, top-8) and picks
  the remaining shapes so the parameter count lands at ~284B total / ~13B
  active.  Every V4-Flash number measured with it is derived from this
  assumption.

Differences between the families are data, not code paths: per-layer
compression ratio, compressor window overlap, indexer ownership, expert weight
format and router score function are all fields.
"""

from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass
from enum import Enum
from pathlib import Path
from typing import Any


class LayerKind(str, Enum):
    """Attention/state-sharing role of one decoder layer.

    Mirrors the reference's layer taxonomy (``config.py:11-21``) and adds the
    V4-Flash roles (every compressed layer owns its compressor there).
    """

    SWA = "swa"                   # sliding window only (r == 0)
    FULL = "full"                 # owns a compressor (kv source) and an indexer
    FULL_CAND = "full_cand"       # FULL + builds the level-1 candidate block mask
    REINDEX = "reindex"           # own indexer over a shared compressed cache
    REUSE = "reuse"               # reuses the latest compressed cache and top-k
    DENSE_COMP = "dense_comp"     # owns a compressor; attends all entries (HCA)
    DSPARK = "dspark"             # MTP draft stage


@dataclass(frozen=True)
class ModelConfig:
    """Complete architecture description (defaults = DeepSeek-V4.1-Flash)."""

    name: str = "deepseek-v4.1-flash"
    family: str = "v4.1"
    vocab_size: int = 129280
    padded_vocab_size: int = 131072
    dim: int = 5120
    n_layers: int = 40
    n_mtp_layers: int = 3
    n_heads: int = 64
    head_dim: int = 512
    qk_rope_head_dim: int = 64
    q_lora_rank: int = 1280
    o_lora_rank: int = 1024
    o_groups: int = 8
    sliding_window: int = 128
    compress_ratios: tuple[int, ...] = (
        0, 0,
        2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2,
        1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1,
        0, 0, 0,
    )
    # Compressor window overlap per layer (1 = pools its own r tokens; 2 = pools
    # the current and the previous group of r tokens).  Empty = all 1.
    compress_overlap: tuple[int, ...] = ()
    # Absolute position embedding added to the compressor gate scores.
    compressor_ape: bool = False
    # Unweighted per-head RMSNorm on q after wq_b (V4-Flash; removed in V4.1).
    q_head_norm: bool = False
    kv_source_layer_ids: tuple[int, ...] = (2, 8, 14, 20)
    index_source_layer_ids: tuple[int, ...] = (2, 8, 14, 20, 24, 28, 32, 36)
    candidate_source_layer_id: int = 20
    candidate_topk_blocks: int = 2048
    candidate_block_size: int = 8
    index_n_heads: int = 32
    index_head_dim: int = 128
    index_topk: int = 512
    rope_theta: float = 10000.0
    compress_rope_theta: float = 160000.0
    rope_factor: float = 16.0
    original_seq_len: int = 65536
    beta_fast: int = 32
    beta_slow: int = 1
    n_routed_experts: int = 384
    n_activated_experts: int = 6
    n_shared_experts: int = 1
    moe_inter_dim: int = 2304
    route_scale: float = 1.5
    score_func: str = "sqrtsoftplus"      # or "sigmoid"
    expert_format: str = "mxfp4"          # "mxfp4" (e2m1 + e8m0/32) or "mxfp8"
    swiglu_limit: float = 10.0
    dspark_n_routed_experts: int = 128
    dspark_n_activated_experts: int = 3
    dspark_block_size: int = 5
    dspark_noise_token_id: int = 128799
    dspark_target_layer_ids: tuple[int, ...] = (37, 38, 39)
    markov_rank: int = 256
    hc_mult: int = 4
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    rms_norm_eps: float = 1e-20
    engram_layer_ids: tuple[int, ...] = (1, 14)
    engram_max_ngram_size: int = 4
    engram_n_heads: int = 8
    engram_head_dim: int = 256
    engram_vocab_size: int = 16000000
    engram_num_embeddings: tuple[int, ...] = (384006168, 384016682)
    engram_pad_id: int = 2
    # "reference": the indexer reads the K cache of the most recent kv-source
    # layer that produced one; "intended": the kv source of this layer.
    index_k_mode: str = "reference"
    eos_token_id: int = 1
    bos_token_id: int = 0

    # ------------------------------------------------------------------ roles
    @property
    def n_total_layers(self) -> int:
        return self.n_layers + self.n_mtp_layers

    def ratio(self, layer_id: int) -> int:
        return self.compress_ratios[layer_id] if layer_id < len(self.compress_ratios) else 0

    def overlap(self, layer_id: int) -> int:
        if not self.compress_overlap:
            return 1
        return self.compress_overlap[layer_id]

    def layer_kind(self, layer_id: int) -> LayerKind:
        if layer_id >= self.n_layers:
            return LayerKind.DSPARK
        r = self.ratio(layer_id)
        if r == 0:
            return LayerKind.SWA
        owns_kv = layer_id in self.kv_source_layer_ids
        owns_idx = layer_id in self.index_source_layer_ids
        if owns_kv and owns_idx:
            return LayerKind.FULL_CAND if layer_id == self.candidate_source_layer_id else LayerKind.FULL
        if owns_kv:
            return LayerKind.DENSE_COMP
        if owns_idx:
            return LayerKind.REINDEX
        return LayerKind.REUSE

    def has_engram(self, layer_id: int) -> bool:
        return layer_id in self.engram_layer_ids

    def kv_source_for(self, layer_id: int) -> int | None:
        """Layer whose compressed KV ``layer_id`` attends (``config.py:102-109``)."""
        if layer_id >= self.n_layers or self.ratio(layer_id) == 0:
            return None
        src = [s for s in self.kv_source_layer_ids if s <= layer_id]
        return src[-1] if src else None

    def index_source_for(self, layer_id: int) -> int | None:
        """Layer whose top-k indices ``layer_id`` reuses (``config.py:111-118``)."""
        if layer_id >= self.n_layers or self.ratio(layer_id) == 0:
            return None
        src = [s for s in self.index_source_layer_ids if s <= layer_id]
        return src[-1] if src else None

    def uses_indexer(self, layer_id: int) -> bool:
        """True if attention of ``layer_id`` selects compressed entries by top-k."""
        return self.index_source_for(layer_id) is not None

    # ------------------------------------------------------------ dimensions
    @property
    def hc_rows(self) -> int:
        return 2 * self.hc_mult + self.hc_mult * self.hc_mult

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def o_inter(self) -> int:
        return self.o_groups * self.o_lora_rank

    @property
    def o_group_in(self) -> int:
        return (self.n_heads // self.o_groups) * self.head_dim

    def n_experts_for(self, layer_id: int) -> int:
        return self.n_routed_experts if layer_id < self.n_layers else self.dspark_n_routed_experts

    def topk_for(self, layer_id: int) -> int:
        return self.n_activated_experts if layer_id < self.n_layers else self.dspark_n_activated_experts

    # ------------------------------------------------------------------ params
    def param_counts(self) -> dict[str, float]:
        """Approximate parameter counts (total, active) in elements."""
        d = self.dim
        attn = (
            d * self.q_lora_rank + self.q_lora_rank * self.q_dim + d * self.head_dim
            + self.o_inter * self.o_group_in + d * self.o_inter + self.hc_rows * self.hc_mult * d * 2
        )
        expert = 3 * d * self.moe_inter_dim
        total = active = 0.0
        for lid in range(self.n_layers):
            comp = 0
            if lid in self.kv_source_layer_ids:
                comp += 2 * self.overlap(lid) * self.head_dim * d
            if lid in self.index_source_layer_ids:
                comp += self.index_n_heads * self.index_head_dim * self.q_lora_rank + self.index_n_heads * d
            dense = attn + comp + self.n_routed_experts * d + self.n_shared_experts * expert
            total += dense + self.n_routed_experts * expert
            active += dense + self.n_activated_experts * expert
        emb = 2 * self.vocab_size * d
        return {"total": total + emb, "active": active + emb}

    # ---------------------------------------------------------------- (de)ser
    def to_dict(self) -> dict[str, Any]:
        return dataclasses.asdict(self)

    @classmethod
    def from_dict(cls, data: dict[str, Any], **overrides: Any) -> "ModelConfig":
        fields = {}
        for f in dataclasses.fields(cls):
            if f.name in data:
                v = data[f.name]
                if isinstance(f.default, tuple) and isinstance(v, list):
                    v = tuple(v)
                fields[f.name] = v
        fields.update(overrides)
        return cls(**fields)

    @classmethod
    def from_json(cls, path: str | Path, **overrides: Any) -> "ModelConfig":
        """Loads a checkpoint ``config.json`` (pattern of ``config.py:120-128``)."""
        return cls.from_dict(json.loads(Path(path).read_text()), **overrides)

    def replace(self, **kw: Any) -> "ModelConfig":
        return dataclasses.replace(self, **kw)


# --------------------------------------------------------------------------
# Named configurations
# --------------------------------------------------------------------------

def v41_flash_config(**overrides: Any) -> ModelConfig:
    """Full DeepSeek-V4.1-Flash: 40 backbone layers + 3 DSpark stages."""
    return ModelConfig(**overrides)


def v41_tiny_config(**overrides: Any) -> ModelConfig:
    """8+2-layer V4.1-shaped config exercising every layer kind and Engram.

    Same layer-role layout as the reference's test config (``config.py:132-176``).
    """
    d = dict(
        name="deepseek-v4.1-tiny",
        vocab_size=1024, padded_vocab_size=1024, dim=256, n_layers=8, n_mtp_layers=2,
        n_heads=32, head_dim=128, qk_rope_head_dim=64, q_lora_rank=128, o_lora_rank=128,
        o_groups=8, sliding_window=16,
        compress_ratios=(0, 0, 2, 2, 2, 1, 1, 1, 0, 0),
        kv_source_layer_ids=(2, 4, 5), index_source_layer_ids=(2, 4, 5, 6),
        candidate_source_layer_id=5, candidate_topk_blocks=8, candidate_block_size=4,
        index_n_heads=32, index_head_dim=64, index_topk=8,
        n_routed_experts=32, n_activated_experts=6, n_shared_experts=1, moe_inter_dim=128,
        dspark_n_routed_experts=16, dspark_n_activated_experts=3, dspark_block_size=5,
        dspark_noise_token_id=1023, dspark_target_layer_ids=(5, 6, 7), markov_rank=64,
        engram_layer_ids=(1, 4), engram_n_heads=8, engram_head_dim=32,
        engram_vocab_size=2048, engram_num_embeddings=(49152, 49152), engram_pad_id=2,
    )
    d.update(overrides)
    return ModelConfig(**d)


def _v4_ratios(n_layers: int) -> tuple[int, ...]:
    # Layers 0-1 sliding window only; then CSA (r=4) and HCA (r=128) alternate.
    return tuple(0 if i < 2 else (4 if i % 2 == 0 else 128) for i in range(n_layers))


def v4_flash_config(**overrides: Any) -> ModelConfig:
    """DeepSeek-V4-Flash-shaped config (dimensions assumed, see module doc).

    * 43 layers, hidden 4096, 64 heads x 512 (64 rope dims), q/o LoRA 1024, 8 o-groups.
    * CSA (r=4, overlapped window, owns an indexer, top-512) alternating with
      HCA (r=128, attends every compressed entry); SWA 128 everywhere.
    * 256 routed experts, top-8, intermediate 2048, 1 shared expert, MXFP8 experts.
    """
    n_layers = overrides.pop("n_layers", 43)
    ratios = _v4_ratios(n_layers)
    kv_src = tuple(i for i, r in enumerate(ratios) if r > 0)
    idx_src = tuple(i for i, r in enumerate(ratios) if r == 4)
    d = dict(
        name="deepseek-v4-flash",
        family="v4",
        vocab_size=129280, padded_vocab_size=131072, dim=4096, n_layers=n_layers, n_mtp_layers=0,
        n_heads=64, head_dim=512, qk_rope_head_dim=64, q_lora_rank=1024, o_lora_rank=1024,
        o_groups=8, sliding_window=128,
        compress_ratios=ratios,
        compress_overlap=tuple(2 if r == 4 else 1 for r in ratios),
        compressor_ape=True, q_head_norm=True,
        kv_source_layer_ids=kv_src, index_source_layer_ids=idx_src,
        candidate_source_layer_id=-1,
        index_n_heads=64, index_head_dim=128, index_topk=512,
        n_routed_experts=256, n_activated_experts=8, n_shared_experts=1, moe_inter_dim=2048,
        route_scale=1.5, score_func="sqrtsoftplus", expert_format="mxfp8",
        engram_layer_ids=(), engram_num_embeddings=(), dspark_target_layer_ids=(),
        # the "reference" K-read quirk belongs to the V4.1 oracle; V4 indexers read their own K
        index_k_mode="intended",
    )
    d.update(overrides)
    cfg = ModelConfig(**d)
    return cfg


def toy_v4_config(**overrides: Any) -> ModelConfig:
    """The CPU/gloo plumbing model: 2 layers, hidden 256, 4 heads x 64, vocab 1024,
    8 experts (inter 128) top-2 sigmoid + 1 shared, ratio-4 compressed attention
    whose indexer keeps 4 blocks of 16 compressed entries (top-64)."""
    d = dict(
        name="toy-v4",
        family="v4",
        vocab_size=1024, padded_vocab_size=1024, dim=256, n_layers=2, n_mtp_layers=0,
        n_heads=4, head_dim=64, qk_rope_head_dim=32, q_lora_rank=128, o_lora_rank=64,
        o_groups=2, sliding_window=16,
        compress_ratios=(4, 4), compress_overlap=(1, 1), compressor_ape=True, q_head_norm=True,
        kv_source_layer_ids=(0, 1), index_source_layer_ids=(0, 1),
        candidate_source_layer_id=-1, candidate_block_size=16,
        index_n_heads=4, index_head_dim=32, index_topk=64,
        n_routed_experts=8, n_activated_experts=2, n_shared_experts=1, moe_inter_dim=128,
        route_scale=1.0, score_func="sigmoid", expert_format="mxfp8",
        engram_layer_ids=(), engram_num_embeddings=(), dspark_target_layer_ids=(), index_k_mode="intended",
    )
    d.update(overrides)
    return ModelConfig(**d)


def v4_check_config(**overrides: Any) -> ModelConfig:
    """Four-layer V4-shaped model at the kernels' dimensions (64 heads x 512 latent,
    64 RoPE dims, 128-wide indexer heads) with overlapped ratio-4 and ratio-16
    compressors and MXFP8 experts: small enough for the CPU oracle, large enough
    that every device kernel path runs.  The verification runner's default."""
    d = dict(name="v4-check", family="v4", vocab_size=1024, padded_vocab_size=1024, dim=512, n_layers=4,
             n_mtp_layers=0, n_heads=64, head_dim=512, qk_rope_head_dim=64, q_lora_rank=256, o_lora_rank=128,
             o_groups=8, sliding_window=16, compress_ratios=(0, 4, 16, 4), compress_overlap=(1, 2, 1, 2),
             compressor_ape=True, q_head_norm=True, kv_source_layer_ids=(1, 2, 3), index_source_layer_ids=(1, 3),
             candidate_source_layer_id=-1, index_n_heads=8, index_head_dim=128, index_topk=8,
             n_routed_experts=16, n_activated_experts=4, n_shared_experts=1, moe_inter_dim=256, route_scale=1.5,
             score_func="sqrtsoftplus", expert_format="mxfp8", engram_layer_ids=(), engram_num_embeddings=(),
             dspark_target_layer_ids=(), index_k_mode="intended")
    d.update(overrides)
    return ModelConfig(**d)


def v41_check_config(**overrides: Any) -> ModelConfig:
    """V4.1-structured model at the kernels' dimensions with two DSpark MTP stages
    (ratio-2 / ratio-1 compressors, 1+4 draft blocks, Markov head): the
    verification runner's speculative-decoding model."""
    d = dict(name="v4.1-check", family="v4.1", vocab_size=1024, padded_vocab_size=1024, dim=512, n_layers=4,
             n_mtp_layers=2, n_heads=64, head_dim=512, qk_rope_head_dim=64, q_lora_rank=256, o_lora_rank=128,
             o_groups=8, sliding_window=16, compress_ratios=(0, 2, 1, 1), kv_source_layer_ids=(1, 2),
             index_source_layer_ids=(1, 2), candidate_source_layer_id=-1, index_n_heads=8, index_head_dim=128,
             index_topk=8, n_routed_experts=16, n_activated_experts=4, n_shared_experts=1, moe_inter_dim=256,
             expert_format="mxfp8", engram_layer_ids=(), engram_num_embeddings=(), index_k_mode="intended",
             dspark_n_routed_experts=8, dspark_n_activated_experts=2, dspark_block_size=5,
             dspark_noise_token_id=1023, dspark_target_layer_ids=(1, 2, 3), markov_rank=128)
    d.update(overrides)
    return ModelConfig(**d)


CONFIGS = {
    "v4.1-flash": v41_flash_config,
    "v4.1-tiny": v41_tiny_config,
    "v4-flash": v4_flash_config,
    "toy-v4": toy_v4_config,
    "v4-check": v4_check_config,
    "v4.1-check": v41_check_config,
}


def get_config(name: str, **overrides: Any) -> ModelConfig:
    if name not in CONFIGS:
        raise KeyError(f"unknown config {name!r}; known: {sorted(CONFIGS)}")
    return CONFIGS[name](**overrides)
