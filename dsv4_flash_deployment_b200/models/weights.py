"""Device weight containers in tensor-core-ready layouts.

Two producers fill the same containers:

* :func:`load_layer` converts reference-checkpoint tensors (names and dtypes of
  ``deepseek_v41/checkpoint.py:73-202``) into kernel layouts: wq_a and wkv are
  fused into one block-scaled weight (one GEMM per token batch), wo_a is
  dequantized to bf16 (its FP8 values are exact in bf16, and the reference
  multiplies it with the bf16 attention output), expert w1/w3 are interleaved
  in 64-row blocks for the SwiGLU epilogue, 32x32 block scales are expanded to
  per-row scale chunks.
* :func:`random_layer` draws the same layouts directly on the device (e4m3
  values ~N(0, 0.5), power-of-two scales 2^-9..2^-5), which is how the
  full-size benchmark models are initialized without a checkpoint.

Expert weights of several layers may share storage (``ExpertStore``): the
1-GPU benchmark cannot hold 256 experts x 43 layers, so layer ``l`` reads the
physical expert block ``l % n_physical``.  Every layer still streams its full
expert bytes from HBM (each block is far larger than L2).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ..ops.gemm import MxWeight, prepare_w13
from ..ops.layout import ceil_to, expand_block_scales
from ..ref import numerics as N


@dataclass
class ExpertBlock:
    w13: MxWeight          # [E_local * 2I, D]
    w2: MxWeight           # [E_local * D, I]
    n_experts: int
    inter: int


@dataclass
class LayerW:
    layer_id: int
    prefix: str
    hc_attn: tuple = ()    # (fn as bf16 hi|lo rows [128, 4D], scale [3], base [24])
    hc_ffn: tuple = ()
    attn_norm: torch.Tensor | None = None
    ffn_norm: torch.Tensor | None = None
    wqkv_a: MxWeight | None = None
    q_norm: torch.Tensor | None = None
    kv_norm: torch.Tensor | None = None
    wq_b: MxWeight | None = None
    wo_a: torch.Tensor | None = None       # bf16 [o_groups * o_lora, o_group_in]
    wo_b: MxWeight | None = None
    sink: torch.Tensor | None = None
    comp_wkvg: torch.Tensor | None = None  # bf16 [2*co*512 (pad 128), D]
    comp_ape: torch.Tensor | None = None
    comp_norm: torch.Tensor | None = None
    idx_wk: torch.Tensor | None = None
    idx_knorm: torch.Tensor | None = None
    idx_wproj: torch.Tensor | None = None  # bf16 [pad128(n_heads), D]
    idx_wq_b: MxWeight | None = None
    gate_w: torch.Tensor | None = None     # bf16 [pad128(E), D]
    gate_b: torch.Tensor | None = None
    experts: ExpertBlock | None = None
    shared_w13: MxWeight | None = None
    shared_w2: MxWeight | None = None
    extra: dict = field(default_factory=dict)


def hc_fn_hilo(fn: torch.Tensor) -> torch.Tensor:
    """fp32 mixing projection [24, 4D] -> bf16 [128, 4D]: rows 0-23 = bf16(fn), rows
    24-47 = bf16(fn - bf16(fn)), rest zero.  hi + lo reproduces fn to ~2^-16 relative,
    so the tensor-core GEMM with fp32 accumulation matches the fp32 projection."""
    fn = fn.float()
    hi = fn.to(torch.bfloat16)
    lo = (fn - hi.float()).to(torch.bfloat16)
    out = torch.zeros(128, fn.shape[1], dtype=torch.bfloat16, device=fn.device)
    out[: fn.shape[0]] = hi
    out[fn.shape[0]: 2 * fn.shape[0]] = lo
    return out


def _hc_params(fn, scale, base, dev):
    return (hc_fn_hilo(fn.to(dev)), scale.float().to(dev).contiguous(), base.float().to(dev).contiguous())


def _pad_rows(w: torch.Tensor, mult: int = 128) -> torch.Tensor:
    n = w.shape[0]
    npad = ceil_to(n, mult)
    if npad == n:
        return w.contiguous()
    out = torch.zeros(npad, *w.shape[1:], dtype=w.dtype, device=w.device)
    out[:n] = w
    return out


def _mx(w, s, dev) -> MxWeight:
    return MxWeight.from_checkpoint(w.to(dev), s.to(dev), dev)


def _cat_mx(parts, dev) -> MxWeight:
    """Concatenate FP8 weights along rows (each part's rows a multiple of 32)."""
    ws = torch.cat([w.view(torch.uint8) for w, _ in parts]).view(torch.float8_e4m3fn)
    ss = torch.cat([expand_block_scales(s, w.shape[0]) for w, s in parts])
    return MxWeight.from_checkpoint(ws.to(dev), ss.to(dev), dev)


def load_layer(cfg, W: dict, lid: int, dev, prefix: str | None = None, experts: ExpertBlock | None = None,
               expert_range: tuple[int, int] | None = None) -> LayerW:
    """Checkpoint tensors -> LayerW for backbone layer ``lid`` (or an MTP stage).

    ``expert_range`` = (first, count) loads only an expert-parallel rank's experts.
    """
    p = prefix or f"layers.{lid}"
    g = lambda k: W[f"{p}.{k}"]
    L = LayerW(layer_id=lid, prefix=p)
    L.hc_attn = _hc_params(g("hc_attn_fn"), g("hc_attn_scale"), g("hc_attn_base"), dev)
    L.hc_ffn = _hc_params(g("hc_ffn_fn"), g("hc_ffn_scale"), g("hc_ffn_base"), dev)
    L.attn_norm = g("attn_norm.weight").to(dev)
    L.ffn_norm = g("ffn_norm.weight").to(dev)
    L.wqkv_a = _cat_mx([(g("attn.wq_a.weight"), g("attn.wq_a.scale")), (g("attn.wkv.weight"), g("attn.wkv.scale"))], dev)
    L.q_norm = g("attn.q_norm.weight").to(dev)
    L.kv_norm = g("attn.kv_norm.weight").to(dev)
    L.wq_b = _mx(g("attn.wq_b.weight"), g("attn.wq_b.scale"), dev)
    L.wo_a = N.dequant_fp8_block(g("attn.wo_a.weight"), g("attn.wo_a.scale")).to(torch.bfloat16).to(dev)
    L.wo_b = _mx(g("attn.wo_b.weight"), g("attn.wo_b.scale"), dev)
    L.sink = g("attn.attn_sink").float().to(dev)
    backbone = lid < cfg.n_layers
    if backbone and lid in cfg.kv_source_layer_ids:
        wkv = g("attn.compressor.wkv.weight")
        wg = W.get(f"{p}.attn.compressor.wgate.weight")
        if wg is None:
            wg = torch.zeros_like(wkv)
        L.comp_wkvg = _pad_rows(torch.cat([wkv, wg])).to(dev)
        ape = W.get(f"{p}.attn.compressor.ape")
        L.comp_ape = ape.float().to(dev).contiguous() if ape is not None else None
        L.comp_norm = g("attn.compressor.norm.weight").to(dev)
    if backbone and lid in cfg.index_source_layer_ids:
        if lid in cfg.kv_source_layer_ids:
            L.idx_wk = g("attn.indexer.wk.weight").to(dev).contiguous()
            L.idx_knorm = g("attn.indexer.k_norm.weight").to(dev)
        L.idx_wproj = _pad_rows(g("attn.indexer.weights_proj.weight")).to(dev)
        L.idx_wq_b = _mx(g("attn.indexer.wq_b.weight"), g("attn.indexer.wq_b.scale"), dev)
    L.gate_w = _pad_rows(g("ffn.gate.weight")).to(dev)
    L.gate_b = g("ffn.gate.bias").float().to(dev)
    if experts is None:
        e0, n_exp = expert_range or (0, cfg.n_experts_for(lid))
        e = lambda i, k: W[f"{p}.ffn.experts.{e0 + i}.{k}"]
        w13s = [prepare_w13(e(i, "w1.weight"), e(i, "w1.scale"), e(i, "w3.weight"), e(i, "w3.scale"), "cpu")
                for i in range(n_exp)]
        w13 = MxWeight(torch.cat([m.q for m in w13s]).to(dev), torch.cat([m.sf for m in w13s]).to(dev),
                       n_exp * w13s[0].n, w13s[0].k, w13s[0].kind)
        w2s = [MxWeight.from_checkpoint(e(i, "w2.weight"), expand_block_scales(e(i, "w2.scale"), cfg.dim), "cpu")
               for i in range(n_exp)]
        w2 = MxWeight(torch.cat([m.q for m in w2s]).to(dev), torch.cat([m.sf for m in w2s]).to(dev),
                      n_exp * w2s[0].n, w2s[0].k, w2s[0].kind)
        experts = ExpertBlock(w13, w2, n_exp, cfg.moe_inter_dim)
    L.experts = experts
    sp = "ffn.shared_experts"
    L.shared_w13 = prepare_w13(g(f"{sp}.w1.weight"), g(f"{sp}.w1.scale"), g(f"{sp}.w3.weight"),
                               g(f"{sp}.w3.scale"), dev)
    L.shared_w2 = _mx(g(f"{sp}.w2.weight"), g(f"{sp}.w2.scale"), dev)
    return L


# ------------------------------------------------------------- random init
def _rand_mx(n: int, k: int, dev, gen: torch.Generator, kind_e2m1: bool = False) -> MxWeight:
    npad = ceil_to(n, 128)
    if kind_e2m1:
        q = torch.randint(0, 256, (npad, k // 2), device=dev, dtype=torch.uint8, generator=gen)
    else:
        q = torch.empty(npad, k, device=dev, dtype=torch.uint8)
        step = max(128, (1 << 28) // k)  # ~1 GB of fp32 scratch per chunk
        for r0 in range(0, npad, step):
            r1 = min(npad, r0 + step)
            q[r0:r1] = (torch.randn(r1 - r0, k, device=dev, generator=gen) * 0.5).to(torch.float8_e4m3fn).view(
                torch.uint8)
    lo = 115 if kind_e2m1 else 118   # e2m1 codes span +-6: scales 3 binades lower match e4m3 magnitudes
    sf = torch.randint(lo, lo + 5, (npad // 128, k // 128, 512), device=dev, dtype=torch.uint8, generator=gen)
    return MxWeight(q, sf, n, k, 2 if kind_e2m1 else 1)


def random_experts(cfg, n_experts: int, dev, gen: torch.Generator, inter: int | None = None) -> ExpertBlock:
    """``inter``: intermediate width per expert (default the model's; a tensor-parallel
    expert split draws each rank's 1/N slice directly)."""
    e2m1 = cfg.expert_format == "mxfp4"
    i, d = inter or cfg.moe_inter_dim, cfg.dim
    w13 = _rand_mx(n_experts * 2 * i, d, dev, gen, e2m1)
    w2 = _rand_mx(n_experts * d, i, dev, gen, e2m1)
    return ExpertBlock(w13, w2, n_experts, i)


def random_layer(cfg, lid: int, dev, gen: torch.Generator, experts: ExpertBlock) -> LayerW:
    d = cfg.dim
    L = LayerW(layer_id=lid, prefix=f"layers.{lid}")

    def bf(n, k):
        return (torch.randn(n, k, device=dev, generator=gen) / k ** 0.5).to(torch.bfloat16)

    def norm(n):
        return (1.0 + 0.05 * torch.randn(n, device=dev, generator=gen)).to(torch.bfloat16)

    def hc():
        fn = torch.randn(cfg.hc_rows, cfg.hc_mult * d, device=dev, generator=gen) * 0.02
        return _hc_params(fn, torch.full((3,), 0.25, device=dev),
                          torch.randn(cfg.hc_rows, device=dev, generator=gen) * 0.05, dev)

    L.hc_attn, L.hc_ffn = hc(), hc()
    L.attn_norm, L.ffn_norm = norm(d), norm(d)
    L.wqkv_a = _rand_mx(cfg.q_lora_rank + cfg.head_dim, d, dev, gen)
    L.q_norm, L.kv_norm = norm(cfg.q_lora_rank), norm(cfg.head_dim)
    L.wq_b = _rand_mx(cfg.q_dim, cfg.q_lora_rank, dev, gen)
    wo_a_q = (torch.randn(cfg.o_inter, cfg.o_group_in, device=dev, generator=gen) * 0.5).to(torch.float8_e4m3fn)
    L.wo_a = (wo_a_q.float() * 2.0 ** -7).to(torch.bfloat16)
    L.wo_b = _rand_mx(d, cfg.o_inter, dev, gen)
    L.sink = torch.randn(cfg.n_heads, device=dev, generator=gen) * 0.1 - 2.0
    if lid in cfg.kv_source_layer_ids:
        co = cfg.overlap(lid)
        r = cfg.ratio(lid)
        L.comp_wkvg = _pad_rows(bf(2 * co * cfg.head_dim, d))
        L.comp_ape = torch.randn(r, co * cfg.head_dim, device=dev, generator=gen) * 0.02 if cfg.compressor_ape else None
        L.comp_norm = norm(cfg.head_dim)
    if lid in cfg.index_source_layer_ids:
        if lid in cfg.kv_source_layer_ids:
            L.idx_wk = bf(cfg.index_head_dim, cfg.head_dim)
            L.idx_knorm = norm(cfg.index_head_dim)
        L.idx_wproj = _pad_rows(bf(cfg.index_n_heads, d))
        L.idx_wq_b = _rand_mx(cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank, dev, gen)
    L.gate_w = _pad_rows(bf(cfg.n_experts_for(lid), d))
    L.gate_b = torch.randn(cfg.n_experts_for(lid), device=dev, generator=gen) * 0.02
    L.experts = experts
    si = cfg.n_shared_experts * cfg.moe_inter_dim
    L.shared_w13 = _rand_mx(2 * si, d, dev, gen)
    L.shared_w2 = _rand_mx(d, si, dev, gen)
    return L
