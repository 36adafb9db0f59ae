"""Grouped MXFP8 expert GEMMs (W13 with the SwiGLU epilogue, W2) by token-tile width.

Builds E experts with a random number of routed rows each (9..63, the spread of
the decode-heavy steps), V4-Flash expert shapes (W13 4096 x 4096, W2 4096 x 2048
per expert, weights larger than L2 at E >= 32), one tile per (expert, 128 output
rows), and times the same tile lists at each requested BN with CUDA events.
BN 32 covers only the first 32 rows of a tile, so its bytes are a lower bound.

    python -m dsv4_flash_deployment_b200.bench.grouped_bench --experts 32 128 256 --bn 32 64 128
"""

from __future__ import annotations

import argparse
import json

import torch

from ..ops import _ext
from ..ops.gemm import EPI_BF16, EPI_SWIGLU, KIND_MX8

D, I = 4096, 2048


def run(E: int, bns: list[int], iters: int = 20, seed: int = 0, copies: int = 1) -> dict:
    ext = _ext.load(required=True)
    dev = "cuda"
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    u8 = torch.uint8
    W13 = [torch.randint(0, 120, (E * 2 * I, D), device=dev, dtype=u8, generator=g) for _ in range(copies)]
    S13 = [torch.full((E * 2 * I // 128, D // 128, 512), 120, device=dev, dtype=u8) for _ in range(copies)]
    W2 = [torch.randint(0, 120, (E * D, I), device=dev, dtype=u8, generator=g) for _ in range(copies)]
    S2 = [torch.full((E * D // 128, I // 128, 512), 120, device=dev, dtype=u8) for _ in range(copies)]
    w13, w2 = W13[0], W2[0]
    rows = torch.randint(9, 64, (E,), generator=torch.Generator().manual_seed(seed)).tolist()
    R = E * 128
    x = torch.randint(0, 120, (R, D), device=dev, dtype=u8, generator=g)
    xsf = torch.full((R // 128, D // 128, 512), 120, device=dev, dtype=u8)
    h = torch.zeros(R, I, device=dev, dtype=u8)
    hsf = torch.zeros(R // 128, I // 128, 512, device=dev, dtype=u8)
    y = torch.empty(R, D, device=dev, dtype=torch.bfloat16)
    rs = torch.ones(R, device=dev)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)
    t13 = i32([[e * 2 * I + mt * 128, e * 128, rows[e], mt * 128] for e in range(E) for mt in range(2 * I // 128)])
    t2 = i32([[e * D + mt * 128, e * 128, rows[e], mt * 128] for e in range(E) for mt in range(D // 128)])
    n13, n2 = i32([len(t13)]), i32([len(t2)])
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = {"experts": E, "rows_mean": round(sum(rows) / E, 2), "weight_copies": copies}
    for bn in bns:
        def f13(i):
            c = i % copies
            ext.gemm(KIND_MX8, EPI_SWIGLU, W13[c], S13[c], x, xsf, None, w13.shape[0], R, D, bn, 1, t13, n13, rs, h,
                     hsf, 10.0, 2 * I, 0, None, None, err, 0, 1, None, None, None)

        def f2(i):
            c = i % copies
            ext.gemm(KIND_MX8, EPI_BF16, W2[c], S2[c], h, hsf, y, w2.shape[0], R, I, bn, 1, t2, n2, None, None, None,
                     0.0, D, D, None, None, err, 0, 1, None, None, None)

        for fn, name, nbytes in ((f13, "w13", w13.numel() + S13[0].numel()), (f2, "w2", w2.numel() + S2[0].numel())):
            for i in range(3):
                fn(i)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for i in range(iters):
                fn(i)
            b.record()
            torch.cuda.synchronize()
            us = a.elapsed_time(b) / iters * 1e3
            out[f"{name}_bn{bn}_us"] = round(us, 1)
            out[f"{name}_bn{bn}_TBs"] = round(nbytes / us / 1e6, 2)
    if int(err.item()) != 0:
        raise RuntimeError(f"device error word {int(err.item()):#x}")
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, nargs="*", default=[32, 128, 256])
    ap.add_argument("--bn", type=int, nargs="*", default=[32, 64, 128])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--copies", type=int, default=1, help="separately allocated weight copies to cycle over")
    a = ap.parse_args(argv)
    for E in a.experts:
        print(json.dumps(run(E, a.bn, a.iters, copies=a.copies)), flush=True)


if __name__ == "__main__":
    main()
