"""Per-op parity of the fused per-token kernels against the fp32 PyTorch oracle
(``ref/numerics.py``), on small shapes, at a bar tighter than whole-model logits:

* the mHC boundary pair (``hc_post`` + ``hc_finish``): stream update, the 24
  mixes after Sinkhorn, the RMS-normed collapse and its MXFP8 quantization;
* ``qkv_post``: q RMSNorm + MXFP8, kv RMSNorm + RoPE + FP8 round trip.

Rounding points follow the oracle; where the kernel's fp32 summation order
differs from torch's, one bf16 ulp is allowed on a small fraction of elements.
"""

import math

import pytest
import torch

from dsv4_flash_deployment_b200.models.weights import hc_fn_hilo
from dsv4_flash_deployment_b200.ops import _ext
from dsv4_flash_deployment_b200.ops.layout import ceil_to, chunks_to_sf
from dsv4_flash_deployment_b200.ref import numerics as N

pytestmark = pytest.mark.gpu

HC = 4


def _ulp_close(out: torch.Tensor, ref: torch.Tensor, max_mismatch: float = 0.01, max_ulps: float = 1.0):
    """bf16 tensors: every element within ``max_ulps`` bf16 ulps of the reference
    (ulp taken at the larger magnitude of the two), and at most ``max_mismatch``
    of them not bit-equal."""
    o, r = out.float().cpu(), ref.float().cpu()
    ulp = torch.maximum(o.abs(), r.abs()).clamp_min(1e-30) * 2.0 ** -7
    assert bool(((o - r).abs() <= max_ulps * ulp + 1e-30).all()), float(((o - r).abs() / ulp).max())
    frac = float((o != r).float().mean())
    assert frac <= max_mismatch, frac


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.float().flatten().cpu(), b.float().flatten().cpu(), dim=0).item()


def _prev_mix(T, g):
    """A valid (pre | post | comb) set: pre, post positive; comb doubly stochastic-ish."""
    m = torch.randn(T, 24, generator=g)
    pre, post, comb = N.hc_split_sinkhorn(m, torch.tensor([0.5, 0.5, 1.0]), torch.zeros(24), HC, 20, 1e-6)
    return torch.cat([pre, post, comb.reshape(T, 16)], -1).float()


@pytest.mark.parametrize("T", [1, 37])
def test_hc_boundary_matches_oracle(T):
    ext = _ext.load(required=True)
    D, iters, hc_eps, norm_eps = 1024, 20, 1e-6, 1e-6
    g = torch.Generator().manual_seed(T)
    X = (torch.randn(T, HC, D, generator=g)).to(torch.bfloat16)
    y = (torch.randn(T, D, generator=g) * 0.5).to(torch.bfloat16)
    prev = _prev_mix(T, g)
    fn = torch.randn(24, HC * D, generator=g) * 0.02
    scale = torch.tensor([0.7, 1.3, 0.9])
    base = torch.randn(24, generator=g) * 0.1
    norm_w = (1.0 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)

    dev = "cuda"
    Xd = X.to(dev).clone()
    prev_d = prev.to(dev)
    mix_out = torch.zeros(T, 24, dtype=torch.float32, device=dev)
    c = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    parts = torch.empty(T * ext.hc_num_slices(D) * 50, dtype=torch.float32, device=dev)
    u = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    Tp = ceil_to(T, 128)
    uq = torch.empty(Tp, D, dtype=torch.uint8, device=dev)
    usf = torch.zeros(Tp // 128, D // 128, 512, dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    fnhl = hc_fn_hilo(fn.to(dev))
    sc, bs, nw = scale.to(dev), base.to(dev), norm_w.to(dev)
    ext.hc_post(Xd, y.to(dev), None, None, 0, prev_d, fnhl, prev_d, 24, c, parts, None, T, None, err)
    ext.hc_finish(Xd, fnhl, sc, bs, prev_d, nw, mix_out, c, parts, u, uq, usf, T, iters, hc_eps, norm_eps)
    torch.cuda.synchronize()
    assert int(err.item()) == 0

    # oracle: X' = post * y + comb^T X, mixes of X', collapse with the handed-over pre
    post = prev[:, HC:2 * HC]
    comb = prev[:, 2 * HC:].reshape(T, HC, HC)
    Xn = N.hc_post(y, X, post, comb)
    _ulp_close(Xd.cpu(), Xn)
    pre_n, post_n, comb_n = N.hc_mixes(Xd.cpu(), fn, scale, base, HC, iters, hc_eps, norm_eps)
    ref_mix = torch.cat([pre_n, post_n, comb_n.reshape(T, 16)], -1)
    torch.testing.assert_close(mix_out.cpu(), ref_mix, rtol=2e-4, atol=2e-5)
    u_ref = N.rms_norm(N.hc_pre(Xd.cpu(), prev[:, :HC]), norm_w, norm_eps)
    # u rounds twice (the bf16 collapse, then the normalized row): two ulps
    _ulp_close(u.cpu(), u_ref, max_mismatch=0.02, max_ulps=2.0)
    # the MXFP8 copy is exactly the oracle quantization of the kernel's own u
    q_ref, s_ref = N.act_quant(u.cpu())
    assert torch.equal(uq[:T].cpu(), q_ref.view(torch.uint8))
    assert torch.equal(chunks_to_sf(usf.cpu(), T, D // 32), s_ref)


@pytest.mark.parametrize("T", [1, 50])
def test_qkv_post_matches_oracle(T):
    from dsv4_flash_deployment_b200.config import v4_flash_config

    ext = _ext.load(required=True)
    cfg = v4_flash_config(n_layers=2)
    qd, kvd, eps = cfg.q_lora_rank, cfg.head_dim, cfg.rms_norm_eps
    g = torch.Generator().manual_seed(100 + T)
    x = (torch.randn(T, qd + kvd, generator=g) * 2.0).to(torch.bfloat16)
    wq = (1.0 + 0.1 * torch.randn(qd, generator=g)).to(torch.bfloat16)
    wk = (1.0 + 0.1 * torch.randn(kvd, generator=g)).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), generator=g, dtype=torch.int32)
    cos, sin = N.layer_rope_tables(cfg, 4096)["yarn"]

    dev = "cuda"
    Tp = ceil_to(T, 128)
    qr_q = torch.empty(Tp, qd, dtype=torch.uint8, device=dev)
    qr_sf = torch.zeros(Tp // 128, qd // 128, 512, dtype=torch.uint8, device=dev)
    kv = torch.empty(T, kvd, dtype=torch.bfloat16, device=dev)
    ext.qkv_post(x.to(dev), qd, kvd, wq.to(dev), wk.to(dev), eps, qr_q, qr_sf, cos.to(dev).contiguous(),
                 sin.to(dev).contiguous(), pos.to(dev), kv, T)
    torch.cuda.synchronize()

    qr = N.rms_norm(x[:, :qd], wq, eps)
    q_ref, s_ref = N.act_quant(qr)
    # codes may differ where the kernel's rsqrt rounds a value across an fp8 boundary
    q_dev = N.act_dequant(qr_q[:T].cpu().view(torch.float8_e4m3fn), chunks_to_sf(qr_sf.cpu(), T, qd // 32))
    q_orc = N.act_dequant(q_ref, s_ref)
    assert _cos(q_dev, q_orc) > 0.99999
    assert float((q_dev != q_orc).float().mean()) < 0.01
    kv_ref = N.act_quant_roundtrip(N.apply_rope(N.rms_norm(x[:, qd:], wk, eps), cos[pos.long()], sin[pos.long()]))
    assert _cos(kv, kv_ref) > 0.99999
    assert float((kv.cpu().float() != kv_ref.float()).float().mean()) < 0.01
    assert math.isfinite(float(kv.float().abs().max()))
