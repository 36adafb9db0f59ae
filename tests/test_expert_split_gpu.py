"""Expert split of the tensor-parallel layout, on one GPU: every "rank" keeps a
1/N slice of each expert's intermediate dimension (``TPGroup.shard_experts``),
runs the grouped W13 (SwiGLU + requant) and W2 GEMMs on its slice with fp32
output, and the N partial rows of a pair must sum to the whole expert's row."""

import pytest
import torch

import dsv4_flash_deployment_b200.ops.gemm as G
from dsv4_flash_deployment_b200.models.weights import ExpertBlock
from dsv4_flash_deployment_b200.ops.layout import ceil_to
from dsv4_flash_deployment_b200.parallel.tp import TPGroup

pytestmark = pytest.mark.gpu


def _ffn(ext, err, ex: ExpertBlock, xq, xsf, rw, starts, counts, rows, D):
    I = ex.inter
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
    y = torch.zeros(rows, D, dtype=torch.float32, device="cuda")
    ext.gemm(ex.w13.kind, G.EPI_SWIGLU, ex.w13.q, ex.w13.sf, xq, xsf, None, ex.w13.q.shape[0], rows, D, 128, 1, t13,
             torch.tensor([len(t13)], dtype=torch.int32, device="cuda"), rw, hq, hsf, 10.0, 2 * I, 0, None,
             None, err, 0, 1, None, None, None)
    ext.gemm(ex.w2.kind, G.EPI_F32, ex.w2.q, ex.w2.sf, hq, hsf, y, ex.w2.q.shape[0], rows, I, 128, 1, t2,
             torch.tensor([len(t2)], dtype=torch.int32, device="cuda"), None, None, None, 0.0, D, D, None, None,
             err, 0, 1, None, None, None)
    return y


@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
@pytest.mark.parametrize("world", [2, 4])
def test_expert_split_partials_sum_to_whole_expert(fmt, world):
    from dsv4_flash_deployment_b200.ref.numerics import pack_e2m1

    E, I, D = 4, 512, 512
    counts = [3, 0, 37, 130]
    g = torch.Generator().manual_seed(5)

    def wt(n, k):
        if fmt == "mxfp4":
            w = pack_e2m1(torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32).to(torch.uint8)).view(torch.int8)
            s = torch.randint(115, 120, (n, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
        else:
            w = (torch.randn(n, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
            s = torch.randint(118, 123, (n, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
        return w, s

    experts = [(wt(I, D), wt(I, D), wt(D, I)) for _ in range(E)]
    w13s = [G.prepare_w13(a[0], a[1], b[0], b[1], "cpu") for a, b, _ in experts]
    w13 = G.MxWeight(torch.cat([m.q for m in w13s]).cuda(), torch.cat([m.sf for m in w13s]).cuda(),
                     E * 2 * I, D, w13s[0].kind)
    w2s = [G.MxWeight.from_checkpoint(c[0], c[1], "cpu") for _, _, c in experts]
    w2 = G.MxWeight(torch.cat([m.q for m in w2s]).cuda(), torch.cat([m.sf for m in w2s]).cuda(), E * D, I,
                    w2s[0].kind)
    whole = ExpertBlock(w13, w2, E, I)
    starts, rows = [], 0
    for c in counts:
        starts.append(rows)
        rows += ceil_to(c, 128)
    x = torch.randn(rows, D, generator=g).to(torch.bfloat16)
    rw = torch.rand(rows, generator=g).cuda()
    xq, xsf = G.quantize(x.cuda())
    ext = G._ext.load()
    err = G.ErrorWord.get("cuda")
    ref = _ffn(ext, err, whole, xq, xsf, rw, starts, counts, rows, D)
    acc = torch.zeros_like(ref)
    for r in range(world):
        part = TPGroup(r, world, None, "cuda", moe="tp").shard_experts(whole)
        assert part.inter == I // world
        acc += _ffn(ext, err, part, xq, xsf, rw, starts, counts, rows, D)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda")
    for st, c in zip(starts, counts):
        if c:
            a, b = acc[st:st + c], ref[st:st + c]
            cos = torch.nn.functional.cosine_similarity(a, b, dim=-1).min().item()
            assert cos > 0.9999, (fmt, world, cos)
            assert (a - b).abs().max().item() <= 1e-3 * b.abs().max().item() + 1e-6
