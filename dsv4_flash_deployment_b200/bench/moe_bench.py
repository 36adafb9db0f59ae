"""MoE-layer microbenchmark over expert parallelism (run under torchrun, one rank per GPU).

The reference's MoE microbench configuration: hidden 4096, 256 routed SwiGLU
experts (intermediate 2048), top-8 sigmoid gating with router logits ~N(0, 1),
one shared expert, bf16 activations quantized on the fly to MXFP8 (e4m3 +
ue8m0 per 32), MXFP8 expert weights; tokens per rank T in {1, 16, 128, 512,
4096}.  One MoE layer of this engine is timed per T, for each expert
transport:

* ``fused`` (the default transport) router top-k fused with the dispatch that
  stores each routed row straight into its owner's expert rows over NVLink,
  the plan, grouped W13 / W2 GEMMs (the shared expert's tiles in the same
  launches) whose W2 epilogue stores each expert row into the source's return
  buffer, and the weighted top-k reduction in the next mHC boundary kernel;
* ``p2p``  router GEMM + top-k, the packing kernel storing (token, expert)
  records straight into each owner's receive buffer over NVLink, plan + unpack,
  grouped W13 (SwiGLU + requant epilogue) / W2 GEMMs, the combine kernel storing
  expert rows back into the source's buffer, the shared expert (overlapping the
  return), and the weighted top-k reduction in the next mHC boundary kernel;
* ``nccl`` the same kernels with ``all_to_all_single`` for both exchanges (the
  baseline).

Device time with CUDA events around CUDA-graph replays, max over ranks.  The
roofline time of the layer on one rank is the largest of: its expert weight
bytes (experts that receive rows) over the measured HBM copy bandwidth, its
FLOPs over the measured bf16 GEMM peak x 2 (MXFP8 runs at twice the bf16 rate),
and its bytes crossing NVLink (dispatch records + returned rows) over the
measured 770 GB/s peer bandwidth; the reported fraction is roofline / measured.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m dsv4_flash_deployment_b200.bench.moe_bench
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

HBM_GBS, BF16_TFLOPS, NVLINK_GBS = 6547.2, 1647.2, 770.0   # measured peaks (B200 pool); NVLink per direction


def moe_cfg():
    from ..config import v4_flash_config

    return v4_flash_config(n_layers=1, compress_ratios=(0,), compress_overlap=(1,), kv_source_layer_ids=(),
                           index_source_layer_ids=(), score_func="sigmoid", n_routed_experts=256,
                           n_activated_experts=8, n_shared_experts=1, moe_inter_dim=2048)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1,16,128,512,4096")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--transports", default="fused,p2p,nccl")
    a = ap.parse_args(argv)

    from ..engine.builder import build_model
    from ..ops.gemm import ErrorWord, quantize
    from ..parallel.ep import EPGroup

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    cfg = moe_cfg()
    Ts = [int(x) for x in a.tokens.split(",")]
    T_max = max(Ts)
    D, I, E, k = cfg.dim, cfg.moe_inter_dim, cfg.n_routed_experts, cfg.n_activated_experts
    results = []
    for transport in a.transports.split(","):
        ep = EPGroup(rank, world, dist.group.WORLD, dev, transport=transport) if world > 1 else None
        m = build_model(cfg, dev, max_tokens=T_max, n_slots=2, max_seq_len=256, seed=3, ep=ep)
        L = m.layers[0]
        g = torch.Generator(device=dev)
        g.manual_seed(100 + rank)
        x = torch.randn(T_max, D, device=dev, generator=g).to(torch.bfloat16)
        m.u[:T_max].copy_(x)
        quantize(m.u[:T_max], m.uq, m.usf)
        m.mixF.zero_()
        m.mixF[:, 4:8] = 1.0                    # post weights: the MoE output enters every stream
        for T in Ts:
            def layer():
                yp, ps, kk, _ = m._moe(L, T)
                m._hc(T, Y=m.shared_y, yperm=yp, pos=ps, topk=kk, prev=m.mixF)

            for _ in range(3):
                layer()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            st = torch.cuda.Stream(dev)
            st.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(st):
                with torch.cuda.graph(graph, stream=st):
                    for _ in range(a.iters):
                        layer()
            torch.cuda.current_stream(dev).wait_stream(st)
            graph.replay()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            ErrorWord.check(dev)
            us = torch.tensor([e0.elapsed_time(e1) / a.iters * 1e3], device=dev)
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
            # roofline of this rank's share: experts that receive rows stream their weights
            ids = m.route[k][0][:T].flatten()
            touched = torch.zeros(E, dtype=torch.int32, device=dev)
            touched.index_fill_(0, ids.long(), 1)
            dist.all_reduce(touched, op=dist.ReduceOp.MAX)
            e_local = E // world
            t_mine = touched.view(world, e_local)[rank].sum() if world > 1 else touched.sum()
            w_bytes = float(t_mine) * 3 * D * I * (1 + 1 / 32) + 3 * D * I * (1 + 1 / 32)   # + shared expert
            flops = 2.0 * T * k * 3 * D * I + 2.0 * T * 3 * D * I + 2.0 * T * D * E
            link = (T * k * (D + D // 32 + 8) + T * k * D * 2) * (world - 1) / world if world > 1 else 0.0
            t_roof = max(w_bytes / (HBM_GBS * 1e3), flops / (2 * BF16_TFLOPS * 1e6), link / (NVLINK_GBS * 1e3))
            results.append({"transport": transport if world > 1 else "local", "tokens_per_rank": T, "world": world,
                            "us": round(us.item(), 1), "roofline_us": round(t_roof, 1),
                            "roofline_fraction": round(t_roof / us.item(), 3),
                            "experts_touched_on_rank": int(t_mine)})
            del graph
            torch.cuda.synchronize()
            dist.barrier()
        del m, ep
        torch.cuda.synchronize()
        dist.barrier()
    if rank == 0:
        for r in results:
            print(json.dumps(r), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
