"""tcgen05 GEMM kernels vs a plain fp32 PyTorch reference of the same op."""

import pytest
import torch

from dsv4_flash_deployment_b200.ops import gemm as G
from dsv4_flash_deployment_b200.ops.layout import chunks_to_sf, ceil_to
from dsv4_flash_deployment_b200.ref import numerics as N

pytestmark = pytest.mark.gpu


def _rand_fp8_weight(n, k, seed, per_row=False):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
    if per_row:
        s = torch.randint(118, 123, (n, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
    else:
        s = torch.randint(118, 123, (n // 32, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
    return w, s


def _close(out, ref, tol=2e-2):
    out = out.float().cpu()
    ref = ref.float().cpu()
    err = (out - ref).abs()
    rel = err.norm() / ref.norm().clamp_min(1e-12)
    assert rel < 5e-3, f"relative error {rel}"
    assert (err <= tol * ref.abs() + 1e-2 * ref.abs().mean()).all(), f"max err {err.max()}"


def test_act_quant_matches_oracle():
    torch.manual_seed(0)
    x = torch.randn(300, 512) * torch.logspace(-3, 2, 512)
    x = x.to(torch.bfloat16)
    q, sf = G.quantize(x.cuda())
    rq, rs = N.act_quant(x)
    assert torch.equal(q[:300].cpu(), rq.view(torch.uint8))
    assert torch.equal(chunks_to_sf(sf.cpu(), 300, 16), rs)


@pytest.mark.parametrize("n_tok", [1, 7, 32, 64, 100, 256, 300])
@pytest.mark.parametrize("splits", [1, 3])
def test_mx8_dense(n_tok, splits):
    n, k = 384, 1024
    w, s = _rand_fp8_weight(n, k, 1)
    torch.manual_seed(n_tok)
    x = torch.randn(n_tok, k).to(torch.bfloat16)
    ref = N.fp8_linear(x, w, s, torch.float32)
    mw = G.MxWeight.from_checkpoint(w, s, "cuda")
    xq, xsf = G.quantize(x.cuda())
    out = torch.empty(n_tok, n, dtype=torch.float32, device="cuda")
    bn = G.pick_bn(n_tok)
    tiles = (mw.q.shape[0] // 128) * ((n_tok + bn - 1) // bn)
    ws = torch.empty(tiles * splits * 128 * bn, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(tiles, dtype=torch.int32, device="cuda")
    G.gemm_mx(xq, xsf, n_tok, mw, out, G.EPI_F32, splits=splits, workspace=ws, counters=cnt)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda")
    _close(out, ref, 1e-3)
    assert int(cnt.sum()) == 0


def test_mx8_bf16_out_bn_sweep():
    n, k = 256, 512
    w, s = _rand_fp8_weight(n, k, 2, per_row=True)
    x = torch.randn(200, k).to(torch.bfloat16)
    ref = N.fp8_linear(x, w, s, torch.float32)
    mw = G.MxWeight.from_checkpoint(w, s, "cuda")
    xq, xsf = G.quantize(x.cuda())
    for bn, nt in ((32, 20), (64, 50), (128, 200), (256, 200)):
        out = torch.zeros(nt, n, dtype=torch.bfloat16, device="cuda")
        G.gemm_mx(xq, xsf, nt, mw, out, G.EPI_BF16, bn=bn)
        torch.cuda.synchronize()
        _close(out, ref[:nt])


def test_bf16_batched_groups():
    g, mg, kg, t = 4, 128, 256, 37
    w = (torch.randn(g * mg, kg) / kg ** 0.5).to(torch.bfloat16)
    x = torch.randn(t, g * kg).to(torch.bfloat16)
    ref = torch.cat([x[:, i * kg:(i + 1) * kg].float() @ w[i * mg:(i + 1) * mg].float().t() for i in range(g)], 1)
    out = torch.empty(t, g * mg, dtype=torch.bfloat16, device="cuda")
    G.gemm_bf16(x.cuda(), w.cuda(), out, groups=g)
    torch.cuda.synchronize()
    _close(out, ref)


@pytest.mark.parametrize("n_tok", [5, 130])
def test_bf16_dense(n_tok):
    n, k = 256, 768
    w = (torch.randn(n, k) / k ** 0.5).to(torch.bfloat16)
    x = torch.randn(n_tok, k).to(torch.bfloat16)
    ref = x.float() @ w.float().t()
    out = torch.empty(n_tok, n, dtype=torch.float32, device="cuda")
    G.gemm_bf16(x.cuda(), w.cuda(), out, f32_out=True)
    torch.cuda.synchronize()
    _close(out, ref, 1e-3)


@pytest.mark.parametrize("splits", [1, 2])
def test_swiglu_epilogue_dense(splits):
    inter, d = 256, 512
    w1, s1 = _rand_fp8_weight(inter, d, 3)
    w3, s3 = _rand_fp8_weight(inter, d, 4)
    x = torch.randn(40, d).to(torch.bfloat16)
    wts = torch.rand(40)
    g = N.fp8_linear(x, w1, s1).float()
    u = N.fp8_linear(x, w3, s3).float()
    h = (N.swiglu_clamped(g, u, 10.0) * wts[:, None]).to(torch.bfloat16)
    rq, rs = N.act_quant(h)
    mw = G.prepare_w13(w1, s1, w3, s3, "cuda")
    xq, xsf = G.quantize(x.cuda())
    hq = torch.zeros(128, inter, dtype=torch.uint8, device="cuda")
    hsf = torch.zeros(1, inter // 128, 512, dtype=torch.uint8, device="cuda")
    G.gemm_mx(xq, xsf, 40, mw, None, G.EPI_SWIGLU, row_scale=wts.cuda(), hq=hq, hsf=hsf, swiglu_limit=10.0,
              splits=splits)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda")
    got = N.act_dequant(hq[:40].cpu().view(torch.float8_e4m3fn), chunks_to_sf(hsf.cpu(), 40, inter // 32))
    want = N.act_dequant(rq, rs)
    # identical up to rare one-ulp e4m3 flips from fp32 summation order
    mism = (got != want).float().mean()
    assert mism < 0.01, mism
    _close(got, want, 0.07)


def test_grouped_mx8():
    # 3 experts, segments padded to 32 rows, W2-style down projection
    e, n, k = 3, 256, 512
    ws = [_rand_fp8_weight(n, k, 10 + i) for i in range(e)]
    counts = [5, 0, 300]
    starts, rows = [], 0
    for c in counts:
        starts.append(rows)
        rows += ceil_to(c, 128) if c else 0
    x = torch.randn(rows, k).to(torch.bfloat16)
    big_w = torch.cat([w for w, _ in ws]).view(torch.uint8)
    big_s = torch.cat([s.repeat_interleave(32, 0) for _, s in ws])
    mw = G.MxWeight.from_checkpoint(big_w.view(torch.float8_e4m3fn), big_s, "cuda")
    xq, xsf = G.quantize(x.cuda())
    bn = 128
    tiles = []
    for ei, (st, c) in enumerate(zip(starts, counts)):
        for t0 in range(0, c, bn):
            for mt in range(n // 128):
                tiles.append([ei * n + mt * 128, st + t0, min(bn, c - t0), mt * 128])
    tl = torch.tensor(tiles, dtype=torch.int32, device="cuda")
    nt = torch.tensor([len(tiles)], dtype=torch.int32, device="cuda")
    out = torch.zeros(rows, n, dtype=torch.bfloat16, device="cuda")
    G._ext.load().gemm(G.KIND_MX8, G.EPI_BF16, mw.q, mw.sf, xq, xsf, out, mw.q.shape[0], rows, k, 256, 1, tl, nt,
                       None, None, None, 0.0, n, n, None, None, G.ErrorWord.get("cuda"), 0, 1, None, None, None)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda")
    for ei, (st, c) in enumerate(zip(starts, counts)):
        if c:
            ref = N.fp8_linear(x[st:st + c], *ws[ei], torch.float32)
            _close(out[st:st + c], ref)


def test_mx4_weights_dense_and_grouped():
    """MXFP4 (e2m1 + ue8m0/32) weights x MXFP8 activations (the V4.1 expert format)."""
    from dsv4_flash_deployment_b200.ref.numerics import pack_e2m1

    n, k, t = 256, 512, 40
    g = torch.Generator().manual_seed(7)
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32).to(torch.uint8)
    w = pack_e2m1(codes).view(torch.int8)
    s = torch.randint(118, 123, (n, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
    x = torch.randn(t, k, generator=g).to(torch.bfloat16)
    ref = N.fp8_linear(x, w, s, torch.float32)
    mw = G.MxWeight.from_checkpoint(w, s, "cuda")
    assert mw.kind == G.KIND_MX4A
    xq, xsf = G.quantize(x.cuda())
    out = torch.empty(t, n, dtype=torch.float32, device="cuda")
    G.gemm_mx(xq, xsf, t, mw, out, G.EPI_F32)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda")
    _close(out, ref, 1e-3)


@pytest.mark.parametrize("fmt", ["mxfp4", "mxfp8"])
def test_grouped_expert_ffn_matches_oracle(fmt):
    """Grouped W13 (SwiGLU + requant epilogue) then grouped W2, vs the oracle expert FFN."""
    from dsv4_flash_deployment_b200.ops.gemm import prepare_w13
    from dsv4_flash_deployment_b200.ref.numerics import pack_e2m1

    E, I, D = 4, 256, 512
    counts = [3, 0, 37, 130]
    g = torch.Generator().manual_seed(11)

    def wt(n, k):
        if fmt == "mxfp4":
            w = pack_e2m1(torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32).to(torch.uint8)).view(torch.int8)
            s = torch.randint(115, 120, (n, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
        else:
            w = (torch.randn(n, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
            s = torch.randint(118, 123, (n, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
        return w, s

    experts = [(wt(I, D), wt(I, D), wt(D, I)) for _ in range(E)]
    w13s = [prepare_w13(a[0], a[1], b[0], b[1], "cpu") for a, b, _ in experts]
    w13 = G.MxWeight(torch.cat([m.q for m in w13s]).cuda(), torch.cat([m.sf for m in w13s]).cuda(),
                     E * 2 * I, D, w13s[0].kind)
    w2s = [G.MxWeight.from_checkpoint(c[0], c[1], "cpu") for _, _, c in experts]
    w2 = G.MxWeight(torch.cat([m.q for m in w2s]).cuda(), torch.cat([m.sf for m in w2s]).cuda(), E * D, I,
                    w2s[0].kind)
    starts, rows = [], 0
    for c in counts:
        starts.append(rows)
        rows += ceil_to(c, 128)
    x = torch.randn(rows, D, generator=g).to(torch.bfloat16)
    rw = torch.rand(rows, generator=g)
    xq, xsf = G.quantize(x.cuda())
    t13, t2 = [], []
    for e, (st, c) in enumerate(zip(starts, counts)):
        for r0 in range(0, c, 128):
            v = min(128, c - r0)
            t13 += [[e * 2 * I + mt * 128, st + r0, v, mt * 128] for mt in range(2 * I // 128)]
            t2 += [[e * D + mt * 128, st + r0, v, mt * 128] for mt in range(D // 128)]
    t13 = torch.tensor(t13, dtype=torch.int32, device="cuda")
    t2 = torch.tensor(t2, dtype=torch.int32, device="cuda")
    hq = torch.zeros(rows, I, dtype=torch.uint8, device="cuda")
    hsf = torch.zeros(rows // 128, I // 128, 512, dtype=torch.uint8, device="cuda")
    y = torch.zeros(rows, D, dtype=torch.bfloat16, device="cuda")
    ext = G._ext.load()
    err = G.ErrorWord.get("cuda")
    ext.gemm(w13.kind, G.EPI_SWIGLU, w13.q, w13.sf, xq, xsf, None, w13.q.shape[0], rows, D, 128, 1, t13,
             torch.tensor([len(t13)], dtype=torch.int32, device="cuda"), rw.cuda(), hq, hsf, 10.0, 2 * I, 0, None,
             None, err, 0, 1, None, None, None)
    ext.gemm(w2.kind, G.EPI_BF16, w2.q, w2.sf, hq, hsf, y, w2.q.shape[0], rows, I, 128, 1, t2,
             torch.tensor([len(t2)], dtype=torch.int32, device="cuda"), None, None, None, 0.0, D, D, None, None,
             err, 0, 1, None, None, None)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda")
    for e, (st, c) in enumerate(zip(starts, counts)):
        if not c:
            continue
        (w1, s1), (w3, s3), (w2_, s2) = experts[e]
        ref = N.expert_ffn(x[st:st + c], w1, s1, w3, s3, w2_, s2, 10.0, rw[st:st + c, None])
        _close(y[st:st + c], ref, 0.05)


@pytest.mark.parametrize("n_tok", [1, 20, 64, 127, 200])
@pytest.mark.parametrize("splits", [2, 4, 8])
def test_cluster_split_k_dense(n_tok, splits):
    """Split-K reduced inside a thread-block cluster over distributed shared memory:
    bf16/f32 outputs match the oracle and the workspace path bit for bit."""
    n, k = 512, 2048
    w, s = _rand_fp8_weight(n, k, 7)
    torch.manual_seed(n_tok + splits)
    x = torch.randn(n_tok, k).to(torch.bfloat16)
    ref = N.fp8_linear(x, w, s, torch.float32)
    mw = G.MxWeight.from_checkpoint(w, s, "cuda")
    xq, xsf = G.quantize(x.cuda())
    out_c = torch.empty(n_tok, n, dtype=torch.float32, device="cuda")
    G.gemm_mx(xq, xsf, n_tok, mw, out_c, G.EPI_F32, splits=splits)
    out_1 = torch.empty(n_tok, n, dtype=torch.float32, device="cuda")
    G.gemm_mx(xq, xsf, n_tok, mw, out_1, G.EPI_F32, splits=1)
    ob = torch.empty(n_tok, n, dtype=torch.bfloat16, device="cuda")
    G.gemm_mx(xq, xsf, n_tok, mw, ob, G.EPI_BF16, splits=splits)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda")
    _close(out_c, ref, 1e-3)
    _close(ob, ref)
    assert torch.allclose(out_c, out_1, rtol=1e-4, atol=1e-4)


def test_cluster_split_k_bf16_and_swiglu():
    n, k = 256, 4096
    torch.manual_seed(3)
    x = torch.randn(60, k).to(torch.bfloat16)
    wb = (torch.randn(n, k) / k ** 0.5).to(torch.bfloat16)
    wp = torch.zeros(n, k, dtype=torch.bfloat16)
    wp[:n] = wb
    ref = x.float() @ wb.float().t()
    out = torch.empty(60, n, dtype=torch.float32, device="cuda")
    G.gemm_bf16(x.cuda(), wp.cuda(), out, f32_out=True, splits=8)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda")
    _close(out, ref, 1e-3)


@pytest.mark.parametrize("n_tok", [40, 100, 127, 300])
@pytest.mark.parametrize("n,k", [(512, 1024), (4096, 4096), (1536, 2048)])
@pytest.mark.parametrize("epi", [G.EPI_F32, G.EPI_BF16])
@pytest.mark.parametrize("splits", [-1, 1])
def test_mx8_dense_256_row_tiles(n_tok, n, k, epi, splits):
    """Dense GEMMs with M % 256 == 0 and 64/128-token tiles run two M=128 MMAs per
    stage (one 256-row weight tile sharing the token tile), with split-K inside a
    cluster (splits=-1: automatic) and without; the result must match the fp32
    reference of the same op."""
    w, s = _rand_fp8_weight(n, k, 5)
    torch.manual_seed(n_tok + n)
    x = torch.randn(n_tok, k).to(torch.bfloat16)
    ref = N.fp8_linear(x, w, s, torch.float32)
    mw = G.MxWeight.from_checkpoint(w, s, "cuda")
    xq, xsf = G.quantize(x.cuda())
    dt = torch.float32 if epi == G.EPI_F32 else torch.bfloat16
    out = torch.empty(n_tok, n, dtype=dt, device="cuda")
    for _ in range(2):   # the second call reuses the resident cluster / stage state
        G.gemm_mx(xq, xsf, n_tok, mw, out, epi, splits=splits)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda")
    _close(out, ref, 1e-3 if epi == G.EPI_F32 else 2e-2)
