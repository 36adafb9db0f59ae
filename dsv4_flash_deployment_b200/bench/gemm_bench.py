"""Microbenchmark of the tcgen05 block-scaled GEMM against cuBLAS bf16.

Times each kernel with CUDA events after warm-up, over a rotation of weight
copies larger than L2 so every launch streams its weights from HBM.  Prints
one JSON line per shape with achieved TB/s (weight+activation bytes) and
TFLOP/s, and the same for ``torch.matmul`` in bf16 as the library baseline.

    python -m dsv4_flash_deployment_b200.bench.gemm_bench
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from ..ops import gemm as G
from ..ops.layout import ceil_to

SHAPES = [
    # (name, out_features, K, tokens)
    ("wq_a/dec1", 1024, 4096, 1),
    ("wq_b/dec1", 32768, 1024, 1),
    ("wo_b/dec1", 4096, 8192, 1),
    ("wq_b/dec64", 32768, 1024, 64),
    ("wqkv_a/127", 1536, 4096, 127),
    ("wq_b/127", 32768, 1024, 127),
    ("wo_b/127", 4096, 8192, 127),
    ("shared_w2/127", 4096, 2048, 127),
    ("expert_w13/16", 4096, 4096, 16),
    ("wo_b/512", 4096, 8192, 512),
    ("wq_b/1024", 32768, 1024, 1024),
    ("square/4096", 4096, 4096, 4096),
    ("square/8192", 8192, 8192, 8192),
]


def _time(fn, iters: int) -> float:
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for i in range(iters):
        fn(i)
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters * 1e3  # us


def run(shapes=SHAPES, iters: int = 20) -> list[dict]:
    dev = torch.device("cuda")
    l2 = 126 * 2 ** 20
    res = []
    for name, n, k, t in shapes:
        wbytes = n * k
        copies = max(2, math.ceil(2 * l2 / wbytes)) if wbytes < 2 * l2 else 1
        ws = []
        for c in range(copies):
            w = (torch.randn(n, k, device=dev) * 0.5).to(torch.float8_e4m3fn)
            s = torch.randint(118, 123, (n // 32, k // 32), device=dev, dtype=torch.int32).to(torch.uint8)
            ws.append(G.MxWeight.from_checkpoint(w, s, dev))
        x = torch.randn(t, k, device=dev).to(torch.bfloat16)
        xq, xsf = G.quantize(x)
        out = torch.empty(t, n, dtype=torch.bfloat16, device=dev)
        bn = G.pick_bn(t)
        tiles = ceil_to(n, 128) // 128 * ((t + bn - 1) // bn)
        # the engine's policy: split-K inside a thread-block cluster for few output tiles
        splits = max(1, min(8, (k // 128) // 2, 148 // max(1, tiles))) if tiles < 100 else 1

        def ours(i):
            G.gemm_mx(xq, xsf, t, ws[i % copies], out, G.EPI_BF16, splits=splits)

        for i in range(3):
            ours(i)
        us = _time(ours, iters)
        G.ErrorWord.check(dev)
        wb16 = [torch.randn(n, k, device=dev).to(torch.bfloat16) for _ in range(max(1, copies // 2))]

        def lib(i):
            torch.matmul(x, wb16[i % len(wb16)].t())

        for i in range(3):
            lib(i)
        us_lib = _time(lib, iters)
        flops = 2.0 * n * k * t
        row = {
            "shape": name, "N_out": n, "K": k, "tokens": t, "bn": bn, "splits": splits,
            "us": round(us, 2), "TBps": round((n * k + t * k) / us / 1e6, 3), "TFLOPs": round(flops / us / 1e6, 1),
            "cublas_bf16_us": round(us_lib, 2), "cublas_TFLOPs": round(flops / us_lib / 1e6, 1),
        }
        print(json.dumps(row), flush=True)
        res.append(row)
        del ws, wb16
        torch.cuda.empty_cache()
    return res


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default=None, help="comma-separated shape names")
    a = ap.parse_args()
    sel = SHAPES if not a.only else [x for x in SHAPES if x[0] in a.only.split(",")]
    run(sel, iters=a.iters)
