"""Per-op parity of the fused per-token kernels against the fp32 PyTorch oracle
(``ref/numerics.py``), on small shapes, at a bar tighter than whole-model logits:

* the mHC boundary pair (``hc_post`` + ``hc_finish``): stream update, the 24
  mixes after Sinkhorn, the RMS-normed collapse and its MXFP8 quantization;
* ``qkv_post``: q RMSNorm + MXFP8, kv RMSNorm + RoPE + FP8 (a KV8 record, decoded here);
* sparse attention over KV8 / KV4 record caches (window + selected compressed rows).

Rounding points follow the oracle; where the kernel's fp32 summation order
differs from torch's, one bf16 ulp is allowed on a small fraction of elements.
"""

import math

import pytest
import torch

from dsv4_flash_deployment_b200.models.kv_format import (ik4_bytes, ik4_decode, kv4_bytes, kv4_decode, kv8_bytes,
                                                         kv8_decode)
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
    kv_rec = torch.empty(T, kv8_bytes(kvd), dtype=torch.uint8, device=dev)
    ext.qkv_post(x.to(dev), qd, kvd, wq.to(dev), wk.to(dev), eps, qr_q, qr_sf, cos.to(dev).contiguous(),
                 sin.to(dev).contiguous(), pos.to(dev), kv_rec, T)
    torch.cuda.synchronize()
    kv = kv8_decode(kv_rec.cpu(), kvd).to(torch.bfloat16)   # exact: the record holds the round trip

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


@pytest.mark.parametrize("T", [1, 19])
def test_engram_gate_matches_oracle(T):
    """Engram gate: per stream s, dot = <h_s * w_s, key_s> * rsqrt(ms(h_s)) * rsqrt(ms(key_s))
    / sqrt(D), g = sigmoid(signed sqrt(dot)), h_s += g * value (ref/model.py ``_engram``)."""
    ext = _ext.load(required=True)
    D, eps = 1024, 1e-6
    g = torch.Generator().manual_seed(7 + T)
    X = torch.randn(T, HC, D, generator=g).to(torch.bfloat16)
    kv = torch.randn(T, (HC + 1) * D, generator=g).to(torch.bfloat16)
    wgt = 1.0 + 0.1 * torch.randn(HC, D, generator=g)
    Xd = X.cuda().clone()
    ext.engram_gate(Xd, kv.cuda(), wgt.cuda().contiguous(), T, eps)
    torch.cuda.synchronize()

    hf = X.float()
    key = kv[:, :HC * D].float().reshape(T, HC, D)
    val = kv[:, HC * D:].float()
    rstd = torch.rsqrt(hf.square().mean(-1) + eps) * torch.rsqrt(key.square().mean(-1) + eps)
    dot = (hf * wgt * key).sum(-1) * rstd * D ** -0.5
    gate = torch.sigmoid(torch.copysign(torch.sqrt(dot.abs().clamp_min(1e-6)), dot))
    ref = (hf + gate[..., None] * val[:, None, :]).to(torch.bfloat16)
    _ulp_close(Xd.cpu(), ref, max_mismatch=0.02)


@pytest.mark.parametrize("r,co", [(4, 2), (16, 1)])
def test_compress_pool_matches_oracle(r, co):
    """Compressor of one prefill chunk at positions 0..T-1: softmax-gated pooling of the
    group's r projections (2r with the overlap: the previous group's first half),
    RMSNorm, RoPE at the group start, e2m1 / e4m3-per-16 round trip; the indexer key
    from the same latent (bf16 GEMV, RMSNorm, RoPE, e2m1 / ue8m0-per-32).  Reference:
    ``ref/model.py`` ``_compressor`` and ``_indexer``."""
    from dsv4_flash_deployment_b200.config import v4_flash_config

    ext = _ext.load(required=True)
    cfg = v4_flash_config(n_layers=2)
    dh, kd, eps = 512, 128, cfg.rms_norm_eps
    T = 4 * r + 3
    g_ = torch.Generator().manual_seed(31 * r + co)
    proj = torch.randn(T, 2 * co * dh, generator=g_)
    ape = torch.randn(r, co * dh, generator=g_) * 0.5
    norm_w = (1.0 + 0.1 * torch.randn(dh, generator=g_)).to(torch.bfloat16)
    wk = (torch.randn(kd, dh, generator=g_) * dh ** -0.5).to(torch.bfloat16)
    k_norm = (1.0 + 0.1 * torch.randn(kd, generator=g_)).to(torch.bfloat16)
    cos, sin = N.layer_rope_tables(cfg, 4096)["yarn"]
    closes = [p for p in range(T) if (p + 1) % r == 0]
    G = len(closes)

    dev = "cuda"
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)
    max_c = 64
    comp = torch.zeros(2, max_c, kv4_bytes(dh), dtype=torch.uint8, device=dev)
    idx = torch.zeros(2, max_c, ik4_bytes(kd), dtype=torch.uint8, device=dev)
    ring = torch.zeros(2, co * r, 2 * co * dh, dtype=torch.float32, device=dev)
    ext.compress_pool(G, i32([G]), i32([0] * G), i32([p // r for p in closes]), i32([0] * G), i32([0] * G), r, co,
                      proj.to(dev), ape.to(dev), ring, norm_w.to(dev), eps, cos.to(dev).contiguous(),
                      sin.to(dev).contiguous(), comp, wk.to(dev), k_norm.to(dev), idx, None)
    torch.cuda.synchronize()

    d = dh
    sc_all = proj[:, co * dh:] + ape[torch.arange(T) % r]
    kv_all = proj[:, :co * dh]
    for gi, p in enumerate(closes):
        g = p // r
        kvs, scs = [], []
        if co == 2:
            for t in range((g - 1) * r, g * r):
                if t >= 0:
                    kvs.append(kv_all[t, :d])
                    scs.append(sc_all[t, :d])
        for t in range(g * r, (g + 1) * r):
            kvs.append(kv_all[t, (co - 1) * d:])
            scs.append(sc_all[t, (co - 1) * d:])
        kv_s, sc_s = torch.stack(kvs), torch.stack(scs)
        pooled = (kv_s * torch.softmax(sc_s, 0)).sum(0)
        latent = N.rms_norm(pooled.to(torch.bfloat16), norm_w, eps)
        c, s = cos[g * r], sin[g * r]
        want = N.fp4_act_quant_roundtrip(N.apply_rope(latent, c, s), 16, "e4m3")
        got = kv4_decode(comp[0, g].cpu(), dh)
        assert _cos(got, want) > 0.9995, (g, _cos(got, want))
        assert float((got.float() != want.float()).float().mean()) < 0.05
        k = N.rms_norm(N.bf16_linear(latent[None], wk), k_norm, eps)
        k_want = N.fp4_act_quant_roundtrip(N.apply_rope(k, c, s), 32, "e8m0")[0]
        k_got = ik4_decode(idx[0, g].cpu(), kd)
        assert _cos(k_got, k_want) > 0.999, (g, _cos(k_got, k_want))


@pytest.mark.parametrize("nsplit", [1, 4])
def test_attention_over_record_caches_matches_oracle(nsplit):
    """Sparse attention of decode tokens over the quantized caches: window rows as
    KV8 records (ring + this step's row), selected compressed rows as KV4 records.
    Oracle: RoPE on q, ``N.sparse_attn`` over the decoded rows in the kernel's row
    order (window ascending, then the selected entries), inverse RoPE on the output
    (``reference.py:172-235``, ``ref/model.py`` ``_attention``)."""
    from dsv4_flash_deployment_b200.config import v4_flash_config
    from dsv4_flash_deployment_b200.models.kv_format import kv4_encode, kv8_encode

    ext = _ext.load(required=True)
    cfg = v4_flash_config(n_layers=2)
    H, dh, W, max_c, k_sel = 64, 512, 128, 300, 200
    g = torch.Generator().manual_seed(17 + nsplit)
    pos = [70, 900, 1500]                      # window partly filled / full
    T = len(pos)
    q = (torch.randn(T, H, dh, generator=g)).to(torch.bfloat16)
    ring_vals = torch.randn(T, W, dh, generator=g) * 0.7
    step_vals = torch.randn(T, dh, generator=g) * 0.7
    comp_vals = torch.randn(T, max_c, dh, generator=g) * 0.7
    sink = torch.randn(H, generator=g)
    cos, sin = N.layer_rope_tables(cfg, 4096)["yarn"]
    sel = torch.stack([torch.randperm(max_c, generator=g)[:k_sel] for _ in range(T)]).to(torch.int32)
    cnt = torch.tensor([k_sel, 150, k_sel], dtype=torch.int32)

    dev = "cuda"
    ring = kv8_encode(ring_vals)                     # [T slots, W, 528]
    step = kv8_encode(step_vals)                     # [T, 528]
    comp = kv4_encode(comp_vals)                     # [T slots, max_c, 288]
    i32 = lambda v: torch.as_tensor(v, dtype=torch.int32).to(dev)
    out = torch.empty(T, H, dh, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(T * nsplit * 64 * 514, dtype=torch.float32, device=dev)
    ext.attention(q.to(dev), cos.to(dev).contiguous(), sin.to(dev).contiguous(), None, False, cfg.rms_norm_eps,
                  step.to(dev), ring.to(dev), comp.to(dev), i32(range(T)), i32(pos), i32(pos), i32(range(T)),
                  sel.to(dev), cnt.to(dev), sink.to(dev), dh ** -0.5, out, ws if nsplit > 1 else None, T, nsplit,
                  None, 0, None)
    torch.cuda.synchronize()

    ring_dec = kv8_decode(ring, dh)
    comp_dec = kv4_decode(comp, dh)
    step_dec = kv8_decode(step, dh)
    for t, p in enumerate(pos):
        rows = []
        for pp in range(max(0, p - W + 1), p + 1):    # window, ascending; this step's row last
            rows.append(step_dec[t] if pp == p else ring_dec[t, pp % W])
        rows += [comp_dec[t, int(ci)] for ci in sel[t, :int(cnt[t])]]
        kv_all = torch.stack(rows)
        qr = N.apply_rope(q[t], cos[p], sin[p])
        idx = torch.arange(kv_all.shape[0])[None, None]
        o = N.sparse_attn(qr[None, None], kv_all[None], sink, idx, dh ** -0.5)[0, 0]
        want = N.apply_rope(o.to(torch.bfloat16), cos[p], sin[p], inverse=True)
        got = out[t].cpu()
        assert _cos(got, want) > 0.9995, (t, _cos(got, want))
        assert float((got.float() - want.float()).abs().max()) < 0.05 * float(want.float().abs().max())


@pytest.mark.parametrize("tile_rows", [32, 64, 256])
def test_expert_tile_rows_layouts_match(tile_rows, monkeypatch):
    """The MoE plan's row layouts (32/64-row tiles in 128-row slots, packed 128 / 256-row
    tiles) give the same logits as the default layout: every expert row is computed
    the same way whatever tile it lands in."""
    from test_model_gpu import small_v4

    from dsv4_flash_deployment_b200.engine.builder import build_model
    from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
    from dsv4_flash_deployment_b200.models.model import SeqChunk, StepMeta
    from dsv4_flash_deployment_b200.ops.gemm import ErrorWord

    cfg = small_v4()
    w = make_random_weights(cfg, seed=3, include_mtp=False)

    def run():
        m = build_model(cfg, "cuda", max_tokens=96, n_slots=4, max_seq_len=128, weights=w)
        out = []
        g = torch.Generator().manual_seed(1)
        for step in range(3):
            if step == 0:
                meta = StepMeta(cfg, [SeqChunk(i, 0, torch.randint(16, 1000, (20 + 7 * i,), generator=g).tolist(),
                                               True) for i in range(3)])
            else:
                meta = StepMeta(cfg, [SeqChunk(i, 19 + 7 * i + step, [int(40 + 11 * i + step)], True)
                                      for i in range(3)])
            m.upload(meta)
            m.forward(meta)
            out.append(m.logits[:3].clone())
        torch.cuda.synchronize()
        ErrorWord.check("cuda")
        return torch.stack(out)

    monkeypatch.delenv("DSV4_EXPERT_TILE_ROWS", raising=False)
    base = run()
    monkeypatch.setenv("DSV4_EXPERT_TILE_ROWS", str(tile_rows))
    other = run()
    assert _cos(base, other) > 0.99999
    assert torch.equal(base.argmax(-1), other.argmax(-1))
