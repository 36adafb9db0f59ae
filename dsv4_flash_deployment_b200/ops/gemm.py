"""Block-scaled and bf16 linear layers on the tcgen05 GEMM kernel.

``MxWeight`` holds a weight in the tensor-core-ready form: e4m3 (or packed
e2m1) values ``[N_pad, K]`` plus scale chunks.  The checkpoint's FP8 32x32
block scales are expanded to per-row-per-32 scales; that is exact because a
32x32 block scale is the same number for every row of the block.

CPU tensors run the torch oracle math instead (used by the CPU tests and the
gloo plumbing run); CUDA tensors always run the extension.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ref import numerics as N
from . import _ext
from .layout import ceil_to, expand_block_scales, interleave_w13, sf_to_chunks

KIND_BF16, KIND_MX8, KIND_MX4A = 0, 1, 2
EPI_BF16, EPI_F32, EPI_SWIGLU = 0, 1, 2


class ErrorWord:
    """Per-device int32 error word every kernel may write (0 = healthy)."""

    _words: dict = {}

    @classmethod
    def get(cls, device) -> torch.Tensor:
        d = torch.device(device)
        if d.type == "cuda" and d.index is None:   # "cuda" and "cuda:<current>" share one word
            d = torch.device("cuda", torch.cuda.current_device())
        key = str(d)
        if key not in cls._words:
            w = torch.zeros(1, dtype=torch.int32, device=device)
            cls._words[key] = w
            if w.is_cuda:
                mod = _ext.load(required=False)
                if mod is not None and getattr(mod, "debug_bounds", False):
                    mod.debug_bounds_attach(w)     # index checks of the debug build report here
        return cls._words[key]

    @classmethod
    def check(cls, device) -> None:
        w = cls.get(device)
        v = int(w.item())
        if v:
            w.zero_()
            code, kid, detail = v & 0xFF, (v >> 8) & 0xFF, (v >> 16) & 0xFFFF
            raise RuntimeError(f"device error word set: code={code} kernel={kid} detail={detail}")


@dataclass
class MxWeight:
    """Quantized weight [N, K]: values + scale chunks (+ dequantized copy on CPU)."""

    q: torch.Tensor          # e4m3 [N_pad, K] (uint8 view) or e2m1 packed int8 [N_pad, K/2]
    sf: torch.Tensor         # uint8 chunks [N_pad/128, K/128, 512]
    n: int
    k: int
    kind: int
    ref_w: torch.Tensor | None = None     # checkpoint tensors kept for the CPU path
    ref_s: torch.Tensor | None = None

    @staticmethod
    def from_checkpoint(w: torch.Tensor, s: torch.Tensor, device=None, keep_ref: bool = False) -> "MxWeight":
        device = device or w.device
        n = w.shape[0]
        e2m1 = w.dtype in (torch.int8, torch.uint8)
        k = w.shape[1] * (2 if e2m1 else 1)
        rows = expand_block_scales(s, n)
        npad = ceil_to(n, 128)
        if e2m1:
            q = torch.zeros(npad, k // 2, dtype=torch.uint8, device=device)
            q[:n] = w.view(torch.uint8).to(device)
        else:
            q = torch.zeros(npad, k, dtype=torch.uint8, device=device)
            q[:n] = w.view(torch.uint8).to(device)
        sf = sf_to_chunks(rows.to(device), npad)
        mw = MxWeight(q, sf, n, k, KIND_MX4A if e2m1 else KIND_MX8)
        if keep_ref or not q.is_cuda:
            mw.ref_w, mw.ref_s = w, s
        return mw


def quantize(x: torch.Tensor, q_out: torch.Tensor | None = None, sf_out: torch.Tensor | None = None):
    """bf16 [T, K] -> (e4m3 bytes [T, K], scale chunks [ceil(T/128), K/128, 512])."""
    t, k = x.shape
    if q_out is None:
        q_out = torch.empty(ceil_to(max(t, 1), 128), k, dtype=torch.uint8, device=x.device)
    if sf_out is None:
        sf_out = torch.empty(ceil_to(max(t, 1), 128) // 128, k // 128, 512, dtype=torch.uint8, device=x.device)
    if x.is_cuda:
        _ext.load().act_quant_mx(x, q_out, sf_out)
    else:
        q, s = N.act_quant(x)
        q_out[:t] = q.view(torch.uint8)
        sf_out.copy_(sf_to_chunks(s, sf_out.shape[0] * 128)[:, : sf_out.shape[1]])
    return q_out, sf_out


def pick_bn(n_tokens: int) -> int:
    """Token-tile width: the smallest covering tile for small batches, 128 (two TMEM
    accumulators, epilogue overlapped) up to 2048 tokens, 256 beyond."""
    if n_tokens <= 32:
        return 32
    if n_tokens <= 64:
        return 64
    if n_tokens <= 2048:
        return 128
    return 256


def gemm_mx(xq: torch.Tensor, xsf: torch.Tensor, n_tokens: int, w: MxWeight, out: torch.Tensor,
            epi: int = EPI_BF16, splits: int = 1, workspace=None, counters=None, row_scale=None,
            hq=None, hsf=None, swiglu_limit: float = 0.0, bn: int | None = None, max_grid: int = 0,
            publish=None) -> torch.Tensor:
    """out[t, :n] = dequant(x) @ dequant(w).T for t < n_tokens (CUDA).
    ``publish``: peer-sync descriptor (``parallel.tp``) published once every tile is stored."""
    bn = bn or pick_bn(n_tokens)
    ext = _ext.load()
    ext.gemm(w.kind, epi, w.q, w.sf, xq, xsf, out if epi != EPI_SWIGLU else None, w.q.shape[0], n_tokens, w.k,
             bn, splits, None, None, row_scale, hq, hsf, swiglu_limit, w.n,
             out.stride(0) if out is not None else 0, workspace, counters, ErrorWord.get(xq.device), max_grid, 1,
             publish, None, None)
    return out


def gemm_bf16(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, f32_out: bool = False, splits: int = 1,
              workspace=None, counters=None, bn: int | None = None, groups: int = 1,
              n_tokens: int | None = None, m_valid: int | None = None, publish=None) -> torch.Tensor:
    """out[t, :N] = x @ w.T with bf16 operands and fp32 accumulation (w rows padded to 128).

    ``groups > 1``: batched mode, w = [G*Mg, Kg] and x = [T, G*Kg]; group g of the
    output (columns g*Mg..) reads x columns g*Kg.. (the grouped ``wo_a``).
    """
    t = x.shape[0] if n_tokens is None else n_tokens
    k = x.shape[1] // groups
    bn = bn or pick_bn(t)
    _ext.load().gemm(KIND_BF16, EPI_F32 if f32_out else EPI_BF16, w, None, x, None, out, w.shape[0], t, k, bn,
                     splits, None, None, None, None, None, 0.0, m_valid or out.shape[1], out.stride(0), workspace,
                     counters, ErrorWord.get(x.device), 0, groups, publish, None, None)
    return out


def linear_mx(x: torch.Tensor, w: MxWeight, out_dtype=torch.bfloat16) -> torch.Tensor:
    """Convenience (allocating) path: act_quant(x) then block-scaled GEMM."""
    if not x.is_cuda:
        return N.fp8_linear(x, w.ref_w, w.ref_s, out_dtype)
    t = x.shape[0]
    xq, xsf = quantize(x)
    out = torch.empty(t, w.n, dtype=out_dtype, device=x.device)
    return gemm_mx(xq, xsf, t, w, out, EPI_F32 if out_dtype == torch.float32 else EPI_BF16)


def prepare_w13(w1: torch.Tensor, s1: torch.Tensor, w3: torch.Tensor, s3: torch.Tensor, device=None) -> MxWeight:
    """Gate/up pair -> one interleaved weight for the SwiGLU-epilogue GEMM."""
    n = w1.shape[0]
    r1 = expand_block_scales(s1, n)
    r3 = expand_block_scales(s3, n)
    w = interleave_w13(w1.view(torch.uint8), w3.view(torch.uint8))
    s = interleave_w13(r1, r3)
    if w1.dtype == torch.float8_e4m3fn:
        w = w.view(torch.float8_e4m3fn)
    else:
        w = w.view(torch.int8)
    return MxWeight.from_checkpoint(w, s, device)
