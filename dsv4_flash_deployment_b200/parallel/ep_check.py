"""Expert-parallel self-check and transport timing (run under torchrun, one rank per GPU).

Every rank builds the same small V4-shaped model (same checkpoint tensors)
twice: once whole on its GPU (the reference) and once expert-parallel over
all ranks.  Each rank steps its own sequences (data-parallel attention) and
the EP logits must match the local model's.  Then the step of every
transport (NCCL all-to-all, NVLink peer stores, and the fused path whose
dispatch stores straight into the owners' expert rows) is timed on the device
(max over ranks):

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m dsv4_flash_deployment_b200.parallel.ep_check

Prints one JSON line per transport on rank 0 and exits non-zero on a mismatch.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def small_cfg(n_layers: int = 3):
    from ..config import ModelConfig

    return ModelConfig(
        name="ep-check", family="v4", vocab_size=1024, padded_vocab_size=1024, dim=1024, n_layers=n_layers,
        n_mtp_layers=0, n_heads=64, head_dim=512, qk_rope_head_dim=64, q_lora_rank=256, o_lora_rank=128,
        o_groups=8, sliding_window=16, compress_ratios=(0,) + (4,) * (n_layers - 1),
        compress_overlap=(1,) + (2,) * (n_layers - 1), compressor_ape=True, q_head_norm=True,
        kv_source_layer_ids=tuple(range(1, n_layers)), index_source_layer_ids=tuple(range(1, n_layers)),
        candidate_source_layer_id=-1, index_n_heads=8, index_head_dim=128, index_topk=8,
        n_routed_experts=32, n_activated_experts=4, n_shared_experts=1, moe_inter_dim=512, route_scale=1.5,
        score_func="sqrtsoftplus", expert_format="mxfp8", engram_layer_ids=(), engram_num_embeddings=(),
        dspark_target_layer_ids=(), index_k_mode="intended")


def _meta(cfg, rank: int, step: int, n_seq: int, plen: int):
    from ..models.model import SeqChunk, StepMeta

    g = torch.Generator().manual_seed(1000 * rank + 7)
    prompts = torch.randint(16, cfg.vocab_size, (n_seq, plen), generator=g).tolist()
    if step == 0:
        return StepMeta(cfg, [SeqChunk(i, 0, prompts[i], True) for i in range(n_seq)])
    return StepMeta(cfg, [SeqChunk(i, plen + step - 1, [(37 * i + 11 * step + rank) % 1000 + 16], True)
                          for i in range(n_seq)])


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--seqs", type=int, default=4)
    ap.add_argument("--plen", type=int, default=40)
    ap.add_argument("--time-tokens", type=int, default=256)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--transports", default="nccl,p2p,fused")
    a = ap.parse_args(argv)

    from ..engine.builder import build_model
    from ..io.checkpoint_spec import make_random_weights
    from ..ops.gemm import ErrorWord
    from .ep import EPGroup

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    cfg = small_cfg()
    w = make_random_weights(cfg, seed=11, include_mtp=False)
    refs = {}   # one-GPU reference per shared-expert form (merged into the grouped GEMMs or not)
    ok = True
    results = {}
    for transport in a.transports.split(","):
        ep = EPGroup(rank, world, dist.group.WORLD, dev, transport=transport)
        m = build_model(cfg, dev, max_tokens=512, n_slots=a.seqs, max_seq_len=512, weights=w, ep=ep)
        # compare against the same rounding: the fused transport carries the shared
        # expert in its grouped GEMMs, the NCCL / p2p exchanges run it separately
        if m.merge_shared not in refs:
            refs[m.merge_shared] = build_model(cfg, dev, max_tokens=512, n_slots=a.seqs, max_seq_len=512,
                                               weights=w, merge_shared=m.merge_shared)
        ref = refs[m.merge_shared]
        worst, agree, total = 1.0, 0, 0
        for s in range(a.steps):
            meta = _meta(cfg, rank, s, a.seqs, a.plen)
            for mod in (ref, m):
                mod.upload(meta, {})
            ids_ref = ref.forward(meta).clone()
            lg_ref = ref.logits[:a.seqs].clone()
            ids = m.forward(meta).clone()
            lg = m.logits[:a.seqs].clone()
            torch.cuda.synchronize()
            ErrorWord.check(dev)
            cos = torch.nn.functional.cosine_similarity(lg.float(), lg_ref.float(), dim=-1).min().item()
            worst = min(worst, cos)
            agree += int((ids == ids_ref).sum())
            total += ids.numel()
        # the expert FFN sums in a different order across ranks: near-identical, not bit-identical
        good = worst > 0.999 and agree >= total - 1
        # device timing of a decode-shaped step of T tokens per rank (graph-free, events, max over ranks)
        from ..models.model import SeqChunk, StepMeta
        T = a.time_tokens
        tm = StepMeta(cfg, [SeqChunk(0, 0, list(range(16, 16 + T)), True)])
        m.upload(tm, {})
        for _ in range(3):
            m.forward(tm)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            m.forward(tm)
        e1.record()
        torch.cuda.synchronize()
        ErrorWord.check(dev)
        ms = torch.tensor([e0.elapsed_time(e1) / a.iters], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        flag = torch.tensor([0 if good else 1], device=dev)
        dist.all_reduce(flag)
        results[transport] = {"transport": transport, "world": world, "min_logit_cos": worst,
                              "token_agree": f"{agree}/{total}", "ok": bool(flag.item() == 0),
                              "step_ms_T%d" % T: round(ms.item(), 4), "layers": cfg.n_layers}
        ok = ok and flag.item() == 0
        del m, ep
        torch.cuda.synchronize()
        dist.barrier()
    if rank == 0:
        for r in results.values():
            print(json.dumps(r), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    raise SystemExit(0 if ok else 1)


if __name__ == "__main__":
    main()
