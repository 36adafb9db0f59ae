"""PyTorch restatement of the model's numerics contract (the CPU oracle).

Every function here states one piece of the DeepSeek-V4 decode math with the
same rounding points as the reference's JAX oracle
(``models/DeepSeekV4.1-Flash-v6e16/tpu-v7x/deepseek_v41/reference.py`` and
``quant.py``, ``rope.py`` beside it).  The CUDA kernels under ``csrc/`` are
tested against these functions, and the CPU execution path of the engine uses
them directly.

Conventions: activations ``bf16``; accumulation ``fp32``; FP8 = ``e4m3fn``;
scale bytes = biased exponents (``ue8m0``), kept as ``uint8`` tensors.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

FP8_MAX = 448.0
ACT_AMAX_FLOOR = 1e-4
FP4_MAX = 6.0
FP4_E8M0_FLOOR = 6.0 * 2.0 ** -126
FP4_E4M3_FLOOR = 6.0 * 2.0 ** -9
E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                            -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


# ----------------------------------------------------------------- scale math
def e8m0_to_f32(s: torch.Tensor) -> torch.Tensor:
    """Biased-exponent byte -> power-of-two float32 (byte 0 gives 2^-127 as 0 -> denorm 0)."""
    return (s.to(torch.int32) << 23).view(torch.float32)


def pow2_ceil_scale(amax: torch.Tensor, inv_max: float) -> tuple[torch.Tensor, torch.Tensor]:
    """``2^ceil(log2(amax*inv_max))`` from IEEE bits (``quant.py:94-107``).

    Returns (scale_f32, biased_exponent_u8); the exponent is clamped to [0, 254].
    """
    prod = (amax.float() * torch.tensor(inv_max, dtype=torch.float32)).contiguous()
    bits = prod.view(torch.int32)
    exp = (bits >> 23) & 0xFF
    man = bits & 0x7FFFFF
    biased = torch.clamp(exp + (man != 0).to(torch.int32), 0, 254)
    return (biased << 23).view(torch.float32), biased.to(torch.uint8)


# ---------------------------------------------------------------- act quant
def act_quant(x: torch.Tensor, block: int = 32) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-``block`` FP8 quantization with ue8m0 scales (``quant.py:110-145``).

    Returns ``(q e4m3 [..., K], scale_u8 [..., K/block])``.
    """
    k = x.shape[-1]
    xf = x.float().reshape(*x.shape[:-1], k // block, block)
    amax = xf.abs().amax(-1).clamp_min(ACT_AMAX_FLOOR)
    s, s_u8 = pow2_ceil_scale(amax, 1.0 / FP8_MAX)
    q = (xf / s[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(x.shape), s_u8


def act_dequant(q: torch.Tensor, s_u8: torch.Tensor, block: int = 32) -> torch.Tensor:
    k = q.shape[-1]
    v = q.float().reshape(*q.shape[:-1], k // block, block) * e8m0_to_f32(s_u8)[..., None]
    return v.reshape(q.shape)


def act_quant_roundtrip(x: torch.Tensor, block: int = 32) -> torch.Tensor:
    """``act_quant(..., inplace=True)``: quantize then dequantize, back to ``x.dtype``."""
    q, s = act_quant(x, block)
    return act_dequant(q, s, block).to(x.dtype)


def _e2m1_codes(xf: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """E2M1 magnitude codes by exact midpoint compare with ties-to-even (``quant.py:212-236``)."""
    ax = xf.abs()
    s = s[..., None]
    mag = ((ax > 0.25 * s).to(torch.int32) + (ax >= 0.75 * s).to(torch.int32)
           + (ax > 1.25 * s).to(torch.int32) + (ax >= 1.75 * s).to(torch.int32)
           + (ax > 2.5 * s).to(torch.int32) + (ax >= 3.5 * s).to(torch.int32)
           + (ax > 5.0 * s).to(torch.int32))
    neg = torch.signbit(xf).to(torch.int32)
    return mag | (neg << 3)


def fp4_act_quant(x: torch.Tensor, block: int = 32, scale_fmt: str = "e8m0"):
    """Per-``block`` E2M1 quantization (``quant.py:285-350``).

    ``scale_fmt='e8m0'`` (block 32): power-of-two scales, returned as u8 exponents.
    ``scale_fmt='e4m3'`` (block 16): ``e4m3(amax/6)`` scales, returned as e4m3.
    Returns ``(codes_u8 [..., K] in 0..15, scale)``.
    """
    k = x.shape[-1]
    xf = x.float().reshape(*x.shape[:-1], k // block, block)
    amax = xf.abs().amax(-1)
    if scale_fmt == "e4m3":
        amax = amax.clamp_min(FP4_E4M3_FLOOR)
        s_q = (amax / FP4_MAX).to(torch.float8_e4m3fn)
        s = s_q.float()
    else:
        amax = amax.clamp_min(FP4_E8M0_FLOOR)
        s, s_q = pow2_ceil_scale(amax, 1.0 / FP4_MAX)
    codes = _e2m1_codes(xf, s)
    return codes.to(torch.uint8).reshape(x.shape), s_q


def fp4_dequant(codes: torch.Tensor, scale: torch.Tensor, block: int) -> torch.Tensor:
    k = codes.shape[-1]
    vals = E2M1_VALUES.to(codes.device)[codes.long()]
    s = scale.float() if scale.dtype == torch.float8_e4m3fn else e8m0_to_f32(scale)
    return (vals.reshape(*codes.shape[:-1], k // block, block) * s[..., None]).reshape(codes.shape)


def fp4_act_quant_roundtrip(x: torch.Tensor, block: int = 32, scale_fmt: str = "e8m0") -> torch.Tensor:
    codes, s = fp4_act_quant(x, block, scale_fmt)
    return fp4_dequant(codes, s, block).to(x.dtype)


def pack_e2m1(codes: torch.Tensor) -> torch.Tensor:
    """Checkpoint packing: byte = low nibble (even k) | high nibble (odd k) << 4 (``quant.py:455-460``)."""
    c = codes.to(torch.uint8).reshape(*codes.shape[:-1], codes.shape[-1] // 2, 2)
    return c[..., 0] | (c[..., 1] << 4)


def unpack_e2m1(packed: torch.Tensor) -> torch.Tensor:
    u = packed.view(torch.uint8)
    return torch.stack([u & 0xF, (u >> 4) & 0xF], -1).reshape(*u.shape[:-1], u.shape[-1] * 2)


# ------------------------------------------------------------ weight dequant
def dequant_fp8_block(w: torch.Tensor, s_u8: torch.Tensor, block: int = 32) -> torch.Tensor:
    """FP8 weight with [block x block] (or [1 x block]) ue8m0 scales -> fp32 (``quant.py:393-411``)."""
    wf = w.float() if w.dtype == torch.float8_e4m3fn else w.view(torch.float8_e4m3fn).float()
    s = e8m0_to_f32(s_u8)
    n, k = wf.shape[-2], wf.shape[-1]
    rep_n = 1 if s.shape[-2] == n else block
    rep_k = 1 if s.shape[-1] == k else block
    s = s.repeat_interleave(rep_n, -2)[..., :n, :].repeat_interleave(rep_k, -1)[..., :k]
    return wf * s


def dequant_mxfp4(packed: torch.Tensor, s_u8: torch.Tensor, block: int = 32) -> torch.Tensor:
    """Packed e2m1 [N, K/2] + ue8m0 [N, K/32] -> fp32 [N, K] (``quant.py:463-484``)."""
    return fp4_dequant(unpack_e2m1(packed), s_u8, block)


def dequant_expert(w: torch.Tensor, s_u8: torch.Tensor) -> torch.Tensor:
    """Dequantize an expert matrix in either MXFP4 (int8 packed) or MXFP8 (e4m3) storage."""
    if w.dtype == torch.float8_e4m3fn:
        return dequant_fp8_block(w, s_u8)
    return dequant_mxfp4(w, s_u8)


# ------------------------------------------------------------------- linears
def fp8_linear(x: torch.Tensor, w: torch.Tensor, s_u8: torch.Tensor,
               out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """act_quant(x) per 32, then block-scaled GEMM in fp32 (``reference.py:127-141``)."""
    q, s = act_quant(x)
    xd = act_dequant(q, s)
    return (xd @ dequant_expert(w, s_u8).t()).to(out_dtype)


def bf16_linear(x: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    y = x.float() @ w.float().t()
    return y.to(out_dtype or x.dtype)


# --------------------------------------------------------------------- norms
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm in fp32, weight rounded through bf16, result in ``x.dtype`` (``reference.py:36-44``)."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return (y * w.to(torch.bfloat16).float()).to(x.dtype)


# ---------------------------------------------------------------------- rope
def rope_inv_freqs(dim: int, original_seq_len: int, base: float, factor: float,
                   beta_fast: int, beta_slow: int) -> torch.Tensor:
    """Inverse frequencies with optional YaRN ramp (``rope.py:33-62``)."""
    idx = torch.arange(0, dim, 2, dtype=torch.float32)
    freqs = 1.0 / (torch.tensor(base, dtype=torch.float32) ** (idx / dim))
    if original_seq_len > 0:
        def corr(rot: float) -> float:
            return dim * math.log(original_seq_len / (rot * 2 * math.pi)) / (2 * math.log(base))
        low = max(math.floor(corr(beta_fast)), 0)
        high = min(math.ceil(corr(beta_slow)), dim - 1)
        ramp = ((torch.arange(dim // 2, dtype=torch.float32) - low) / max(high - low, 1e-3)).clamp(0, 1)
        smooth = 1.0 - ramp
        freqs = freqs / factor * (1.0 - smooth) + freqs * smooth
    return freqs


def rope_table(dim: int, seqlen: int, original_seq_len: int, base: float, factor: float,
               beta_fast: int, beta_slow: int) -> tuple[torch.Tensor, torch.Tensor]:
    freqs = rope_inv_freqs(dim, original_seq_len, base, factor, beta_fast, beta_slow)
    ang = torch.outer(torch.arange(seqlen, dtype=torch.float32), freqs)
    return torch.cos(ang), torch.sin(ang)


def layer_rope_tables(cfg, seqlen: int) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    """``swa`` table (theta 10000, no YaRN) for r == 0 layers, ``yarn`` for r > 0 (``rope.py:118-141``)."""
    rd = cfg.qk_rope_head_dim
    return {
        "swa": rope_table(rd, seqlen, 0, cfg.rope_theta, cfg.rope_factor, cfg.beta_fast, cfg.beta_slow),
        "yarn": rope_table(rd, seqlen, cfg.original_seq_len, cfg.compress_rope_theta,
                           cfg.rope_factor, cfg.beta_fast, cfg.beta_slow),
    }


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """Interleaved (GPT-J) rotation of the last ``2*cos.shape[-1]`` dims, fp32 math.

    ``cos``/``sin`` broadcast against ``x[..., :half]`` after a head axis is
    inserted by the caller where needed.
    """
    half = cos.shape[-1]
    rd = 2 * half
    tail = x[..., -rd:].float()
    xe, xo = tail[..., 0::2], tail[..., 1::2]
    s = -sin if inverse else sin
    ye = xe * cos - xo * s
    yo = xe * s + xo * cos
    rot = torch.stack([ye, yo], -1).reshape(tail.shape).to(x.dtype)
    if x.shape[-1] == rd:
        return rot
    return torch.cat([x[..., :-rd], rot], -1)


# ----------------------------------------------------------------------- mHC
def hc_split_sinkhorn(mixes: torch.Tensor, scale: torch.Tensor, base: torch.Tensor,
                      hc: int, iters: int, eps: float):
    """Mixes [..., 24] -> (pre [..., hc], post [..., hc], comb [..., hc, hc]) (``reference.py:47-79``)."""
    m = mixes.float()
    s = scale.float()
    b = base.float()
    pre = torch.sigmoid(m[..., :hc] * s[0] + b[:hc]) + eps
    post = 2.0 * torch.sigmoid(m[..., hc:2 * hc] * s[1] + b[hc:2 * hc])
    comb = (m[..., 2 * hc:] * s[2] + b[2 * hc:]).reshape(*m.shape[:-1], hc, hc)
    if iters > 0:
        comb = torch.softmax(comb, -1) + eps
        comb = comb / (comb.sum(-2, keepdim=True) + eps)
        for _ in range(iters - 1):
            comb = comb / (comb.sum(-1, keepdim=True) + eps)
            comb = comb / (comb.sum(-2, keepdim=True) + eps)
    return pre, post, comb


def hc_mixes(x: torch.Tensor, fn: torch.Tensor, scale: torch.Tensor, base: torch.Tensor,
             hc: int, iters: int, eps: float, norm_eps: float):
    """x [..., hc, D] -> (pre, post, comb) (``reference.py:81-103``)."""
    xf = x.reshape(*x.shape[:-2], x.shape[-2] * x.shape[-1]).float()
    r = torch.rsqrt(xf.square().mean(-1, keepdim=True) + norm_eps)
    mixes = (xf @ fn.float().t()) * r
    return hc_split_sinkhorn(mixes, scale, base, hc, iters, eps)


def hc_pre(x: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    """Collapse [..., hc, D] with weights [..., hc] -> [..., D] (``reference.py:105-110``)."""
    return (pre[..., None].float() * x.float()).sum(-2).to(x.dtype)


def hc_post(y: torch.Tensor, residual: torch.Tensor, post: torch.Tensor, comb: torch.Tensor) -> torch.Tensor:
    """new[j] = post[j]*y + sum_i comb[i,j]*res[i] (``reference.py:112-125``)."""
    out = post[..., None].float() * y[..., None, :].float() + (
        comb[..., None].float() * residual[..., :, None, :].float()).sum(-3)
    return out.to(y.dtype)


# ----------------------------------------------------------- sparse attention
def sparse_attn(q: torch.Tensor, kv: torch.Tensor, sink: torch.Tensor, idx: torch.Tensor,
                scale: float) -> torch.Tensor:
    """Sparse MQA over gathered latent rows (K == V), sink in the denominator.

    q [B, M, H, D]; kv [B, N, D]; idx [B, M, K] (-1 = masked). Online softmax over
    blocks of 64 indices with P rounded to bf16 before PV (``reference.py:172-235``).
    """
    b, m, h, d = q.shape
    kk = idx.shape[-1]
    blk = 64
    nb = (kk + blk - 1) // blk
    pad = nb * blk - kk
    if pad:
        idx = F.pad(idx, (0, pad), value=-1)
    qf = q.to(torch.bfloat16).float()
    kvb = kv.to(torch.bfloat16).float()
    acc = torch.zeros(b, m, h, d)
    ssum = torch.zeros(b, m, h)
    smax = torch.full((b, m, h), -1e30)
    bidx = torch.arange(b)[:, None, None]
    for t in range(nb):
        bi = idx[:, :, t * blk:(t + 1) * blk].long()
        valid = bi != -1
        rows = kvb[bidx, bi.clamp_min(0)] * valid[..., None]
        s = torch.einsum("bmhd,bmkd->bmhk", qf, rows) * scale
        s = s.masked_fill(~valid[:, :, None, :], float("-inf"))
        new_max = torch.maximum(smax, s.amax(-1))
        corr = torch.exp(smax - new_max)
        p = torch.exp(s - new_max[..., None])
        ssum = ssum * corr + p.sum(-1)
        acc = acc * corr[..., None] + torch.einsum(
            "bmhk,bmkd->bmhd", p.to(torch.bfloat16).float(), rows)
        smax = new_max
    ssum = ssum + torch.exp(sink.float().reshape(1, 1, h) - smax)
    return (acc / ssum[..., None]).to(q.dtype)


def select_candidate_blocks(scores: torch.Tensor, compress_len, topk_blocks: int, block: int) -> torch.Tensor:
    """Level-1 candidate mask: block max, force the last block, keep top blocks (``reference.py:237-269``)."""
    width = scores.shape[-1]
    pad = (-width) % block
    s = scores.float()
    if pad:
        s = F.pad(s, (0, pad), value=float("-inf"))
    bs = s.reshape(*s.shape[:-1], -1, block).amax(-1)
    nb = bs.shape[-1]
    last = (torch.as_tensor(compress_len) - 1) // block
    ar = torch.arange(nb)
    bs = torch.where(ar == (last[..., None] if last.ndim else last), torch.tensor(float("inf")), bs)
    k = min(topk_blocks, nb)
    vals, ids = torch.topk(bs, k, -1)
    keep = torch.zeros_like(bs, dtype=torch.bool)
    keep.scatter_(-1, ids, vals > float("-inf"))
    return keep.repeat_interleave(block, -1)[..., :width]


# ----------------------------------------------------------------------- MoE
def router_scores(logits: torch.Tensor, score_func: str) -> torch.Tensor:
    if score_func == "sigmoid":
        return torch.sigmoid(logits)
    sp = torch.where(logits > 20.0, logits, torch.log1p(torch.exp(logits)))
    return torch.sqrt(sp)


def route(x: torch.Tensor, gate_w: torch.Tensor, gate_b: torch.Tensor, topk: int,
          route_scale: float, score_func: str) -> tuple[torch.Tensor, torch.Tensor]:
    """Scores -> top-k on score+bias -> normalized weights * route_scale (``reference.py:355-382``)."""
    logits = x.float() @ gate_w.float().t()
    scores = router_scores(logits, score_func)
    _, ids = torch.topk(scores + gate_b.float()[None], topk, -1)
    w = scores.gather(-1, ids)
    if topk > 1:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return ids, w * route_scale


def swiglu_clamped(gate: torch.Tensor, up: torch.Tensor, limit: float) -> torch.Tensor:
    g = gate.float()
    u = up.float()
    if limit > 0:
        u = u.clamp(-limit, limit)
        g = g.clamp_max(limit)
    return F.silu(g) * u


def expert_ffn(x: torch.Tensor, w1, s1, w3, s3, w2, s2, limit: float,
               weight: torch.Tensor | None = None) -> torch.Tensor:
    """One SwiGLU expert on quantized weights (``reference.py:327-352``); fp32 result."""
    g = fp8_linear(x, w1, s1).float()
    u = fp8_linear(x, w3, s3).float()
    h = swiglu_clamped(g, u, limit)
    if weight is not None:
        h = weight.float() * h
    return fp8_linear(h.to(torch.bfloat16), w2, s2).float()
