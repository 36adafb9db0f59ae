"""DSpark speculative decoding on the GPU: MTP drafter + lossless 1+4 verify.

Per round, for every decoding sequence (reference: ``forward_spec``
reference.py:1116-1248, ``verify_block`` :1250-1329, the v7x drafter
``tpu-v7x/deepseek_v41/dspark.py:271-767``):

  draft   a block [root, noise x (B-1)] at positions d0..d0+B-1 runs through
          the MTP stages mtp.0..K-1 (each a full block: mHC, attention over the
          stage's ring of main-hidden keys plus every row of the draft block,
          MoE with the stage's experts), the shared head, then the Markov head
          chain tok_{i+1} = argmax(logits_i + memb[tok_i] @ mhead^T)
  verify  the target model runs [root, d1..d_{B-1}] as one chunk with logits
          at every position, rings deferred; n_acc = longest prefix with
          pred_i == d_{i+1} (or the forced value); the sequence emits
          d1..d_nacc + pred_nacc
  commit  the rings take only the accepted prefix (positions d0..d0+n_acc);
          position-indexed caches are rewritten before anything reads them
  ingest  main_hidden (mean of the 4 streams entering each tap layer) of the
          accepted rows -> main_proj -> RMSNorm -> per stage wkv -> kv norm ->
          RoPE -> FP8 (KV8 record) -> the stage's ring

Every step reuses the target model's device buffers; only the MTP rings, the
tap buffers and a few small work arrays are added.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from ..models.kv_format import kv8_bytes
from ..models.model import SeqChunk, StepMeta
from ..models.weights import load_layer
from ..ops.gemm import MxWeight, quantize
from ..ops.layout import ceil_to


def _pad_rows(w: torch.Tensor, mult: int = 128) -> torch.Tensor:
    n = w.shape[0]
    p = ceil_to(n, mult)
    if p == n:
        return w.contiguous()
    out = torch.zeros((p,) + tuple(w.shape[1:]), dtype=w.dtype, device=w.device)
    out[:n] = w
    return out


@dataclass
class SpecStats:
    rounds: int = 0
    drafted: int = 0
    accepted: int = 0
    emitted: int = 0
    histogram: list = field(default_factory=list)

    def as_dict(self) -> dict:
        acc_len = self.emitted / max(1, self.rounds)
        return {"rounds": self.rounds, "drafted": self.drafted, "accepted": self.accepted,
                "emitted": self.emitted, "mean_tokens_per_round": acc_len, "histogram": list(self.histogram)}


class DSparkDrafter:
    """MTP stages, Markov head and the per-stage main-hidden rings on the device."""

    def __init__(self, model, weights: dict | None, max_seqs: int, seed: int = 0):
        """``weights``: checkpoint dict (``mtp.*`` names); None draws random stage
        weights on the device (full-size benchmark runs without a checkpoint)."""
        cfg = model.cfg
        if cfg.n_mtp_layers < 1 or not cfg.dspark_target_layer_ids:
            raise ValueError("config has no DSpark stages")
        if getattr(model, "tp", None) is not None:
            raise NotImplementedError("DSpark drafting runs on a whole (not tensor-parallel) backbone")
        self.m, self.cfg, dev = model, cfg, model.dev
        self.ext = model.ext
        self.blk = cfg.dspark_block_size
        self.K = cfg.n_mtp_layers
        if weights is None:
            self._random_init(seed)
        else:
            self.stages = [load_layer(cfg, weights, cfg.n_layers + k, dev, prefix=f"mtp.{k}")
                           for k in range(self.K)]
            self.main_proj = MxWeight.from_checkpoint(weights["mtp.0.main_proj.weight"].to(dev),
                                                      weights["mtp.0.main_proj.scale"].to(dev), dev)
            self.main_norm = weights["mtp.0.main_norm.weight"].to(dev)
            last = f"mtp.{self.K - 1}"
            self.final_norm = weights[f"{last}.norm.weight"].to(dev)
            self.memb = weights[f"{last}.markov_head.embed.weight"].to(dev, torch.bfloat16).contiguous()
            self.mhead = _pad_rows(weights[f"{last}.markov_head.head.weight"].to(dev, torch.bfloat16))
            self.conf_w = weights[f"{last}.confidence_head.proj.weight"].float().to(dev)
        self.R = self.memb.shape[1]
        S = model.n_slots + 1
        W = cfg.sliding_window
        # KV8 records, like the target model's window rings (models/kv_format.py)
        self.rings = [torch.zeros(S, W, kv8_bytes(cfg.head_dim), dtype=torch.uint8, device=dev) for _ in range(self.K)]
        T = model.max_tokens
        D = cfg.dim
        nt = len(cfg.dspark_target_layer_ids)
        self.taps = {lid: torch.zeros(T, D, dtype=torch.bfloat16, device=dev) for lid in cfg.dspark_target_layer_ids}
        self.mh = torch.zeros(T, nt * D, dtype=torch.bfloat16, device=dev)
        self.mx = torch.zeros(T, D, dtype=torch.bfloat16, device=dev)
        self.kvraw = torch.zeros(T, cfg.head_dim, dtype=torch.bfloat16, device=dev)
        self.kvq = torch.zeros(T, kv8_bytes(cfg.head_dim), dtype=torch.uint8, device=dev)
        n = max_seqs
        self.toks = torch.zeros(self.blk + 1, n, dtype=torch.int32, device=dev)
        self.emb = torch.zeros(n, self.R, dtype=torch.bfloat16, device=dev)
        self.mlog = torch.zeros(n, self.mhead.shape[0], dtype=torch.float32, device=dev)
        self.dummy_q = torch.zeros(ceil_to(T, 128), 128, dtype=torch.uint8, device=dev)
        self.dummy_sf = torch.zeros(ceil_to(T, 128) // 128, 1, 512, dtype=torch.uint8, device=dev)

    def _random_init(self, seed: int) -> None:
        """Stage layers (each with its own expert block), main_proj, norms and the
        Markov / confidence heads drawn on the device, in the checkpoint layouts."""
        from ..models.weights import _rand_mx, random_experts, random_layer

        cfg, dev = self.cfg, self.m.dev
        g = torch.Generator(device=dev)
        g.manual_seed(seed + 777)
        D, V, R = cfg.dim, cfg.vocab_size, cfg.markov_rank
        self.stages = []
        for k in range(self.K):
            lid = cfg.n_layers + k
            ex = random_experts(cfg, cfg.n_experts_for(lid), dev, g)
            self.stages.append(random_layer(cfg, lid, dev, g, ex))
        nt = len(cfg.dspark_target_layer_ids)
        self.main_proj = _rand_mx(D, nt * D, dev, g)
        norm = lambda n: (1.0 + 0.05 * torch.randn(n, device=dev, generator=g)).to(torch.bfloat16)
        self.main_norm, self.final_norm = norm(D), norm(D)
        self.memb = (torch.randn(V, R, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.mhead = _pad_rows((torch.randn(V, R, device=dev, generator=g) / R ** 0.5).to(torch.bfloat16))
        self.conf_w = torch.randn(1, D + R, device=dev, generator=g) * 0.02

    # ----------------------------------------------------------------- ingest
    def ingest(self, rows: torch.Tensor | None, T: int) -> None:
        """main_hidden rows -> every stage ring, for the metadata currently uploaded.

        ``rows``: [T] int64 device indices of the rows to take from the tap
        buffers (None = rows 0..T-1 in order).
        """
        m, cfg, ext = self.m, self.cfg, self.ext
        D = cfg.dim
        for i, lid in enumerate(cfg.dspark_target_layer_ids):
            src = self.taps[lid][:T] if rows is None else self.taps[lid].index_select(0, rows)
            self.mh[:T, i * D:(i + 1) * D].copy_(src)
        q, sf = quantize(self.mh[:T])
        m._gemm(q, sf, T, self.main_proj, self.mx)
        # main_x = RMSNorm(main_proj(main_hidden)) -> MXFP8 for the per-stage wkv GEMMs
        x = self.mx[:T].float()
        x = (x * torch.rsqrt(x.square().mean(-1, keepdim=True) + cfg.rms_norm_eps) *
             self.main_norm.float()).to(torch.bfloat16)
        xq, xsf = quantize(x)
        cos, sin = m.rope["swa"]
        for k, L in enumerate(self.stages):
            # rows of wqkv_a past q_lora_rank are wkv: run the fused weight, keep the kv part
            qkv = torch.empty(T, cfg.q_lora_rank + cfg.head_dim, dtype=torch.bfloat16, device=m.dev)
            m._gemm(xq, xsf, T, L.wqkv_a, qkv)
            self.kvraw[:T].copy_(qkv[:, cfg.q_lora_rank:])
            ext.qkv_post(self.kvraw, 0, cfg.head_dim, L.kv_norm, L.kv_norm, cfg.rms_norm_eps, self.dummy_q,
                         self.dummy_sf, cos, sin, m.m_pos, self.kvq, T)
            ext.ring_update(self.rings[k], self.kvq, T, m.m_slot, m.m_pos, m.m_last)

    # ------------------------------------------------------------------ draft
    def draft(self, n: int) -> torch.Tensor:
        """Runs the uploaded draft metadata (n sequences x block rows); fills self.toks.

        ``self.toks[0, :n]`` must hold the roots.  Returns toks [blk+1, n] (device).
        """
        m, cfg, ext = self.m, self.cfg, self.ext
        T = n * self.blk
        meta = m._last_meta
        ext.embed_streams(m.embed, m.m_ids, T, m.X)
        moe_state = None
        win = cfg.sliding_window + self.blk
        for k, L in enumerate(self.stages):
            if moe_state is None:
                m._hc(T, prev=None, mixes=L.hc_attn, cw=m.mix0, norm=L.attn_norm, mix_out=m.mixA, u=m.u, uq=m.uq,
                      usf=m.usf)
            else:
                yp, ps, kk, _ = moe_state
                m._hc(T, Y=m.shared_y, yperm=yp, pos=ps, topk=kk, prev=m.mixF, mixes=L.hc_attn, cw=m.mixF,
                      norm=L.attn_norm, mix_out=m.mixA, u=m.u, uq=m.uq, usf=m.usf)
            m._attention(L, meta, ring=self.rings[k], win_len=win)
            m._hc(T, Y=m.attn_out, prev=m.mixA, mixes=L.hc_ffn, cw=m.mixA, norm=L.ffn_norm, mix_out=m.mixF, u=m.u,
                  uq=m.uq, usf=m.usf)
            moe_state = m._moe(L, T)
        yp, ps, kk, _ = moe_state
        m._hc(T, Y=m.shared_y, yperm=yp, pos=ps, topk=kk, prev=m.mixF, mixes=None, cw=m.mixF,
              norm=self.final_norm, u=m.u)
        m._gemm_bf16(m.u[:T], m.head, m.logits[:T], T, f32_out=True)
        V = m.vocab
        ext.markov_step(m.logits, self.blk, -1, self.mlog, V, n, self.toks, self.memb, self.emb)
        for i in range(self.blk):
            m._gemm_bf16(self.emb[:n], self.mhead, self.mlog[:n], n, f32_out=True)
            ext.markov_step(m.logits, self.blk, i, self.mlog, V, n, self.toks, self.memb, self.emb)
        return self.toks[:, :n]


class SpecEngine:
    """Greedy generation with DSpark drafts and lossless verification (single GPU).

    ``force_accept``: accept exactly this many drafts per round regardless of
    agreement (the reference's knob for random-weight runs, engine.py:332);
    outputs then differ from greedy, the acceptance path is exercised.  A
    fractional value f accepts floor(f) or ceil(f) drafts per round in a fixed
    pattern whose mean is f (e.g. 2.15 reproduces the reference's measured
    3.15 tokens per round, ``MK/results/megakernel_v6e16_results.json:777``).
    """

    def __init__(self, model, weights: dict | None, max_seqs: int = 16, force_accept: int | None = None):
        self.m = model
        self.cfg = model.cfg
        self.drafter = DSparkDrafter(model, weights, max_seqs)
        self.blk = self.cfg.dspark_block_size
        self.force_accept = force_accept
        self._forced_rounds = 0
        self.stats = SpecStats(histogram=[0] * self.blk)
        self.max_seqs = max_seqs
        self.pinned: dict = {}

    def _run(self, meta: StepMeta, **kw) -> torch.Tensor:
        m = self.m
        m.upload(meta, self.pinned)
        m._last_meta = meta
        taps = kw.pop("taps", None)
        return m.forward(meta, taps=taps, **kw)

    def _ingest_meta(self, seqs, rows_per_seq, starts) -> StepMeta:
        return StepMeta(self.cfg, [SeqChunk(s, st, [0] * r, False) for s, r, st in zip(seqs, rows_per_seq, starts)])

    # ------------------------------------------------------------ phases
    def prefill(self, prompts: list[list[int]]) -> None:
        """Prefills each prompt (chunked), fills the MTP rings; sets the first token."""
        m, cfg, dr = self.m, self.cfg, self.drafter
        if len(prompts) > self.max_seqs:
            raise ValueError("too many sequences for the drafter's buffers")
        self.slots = list(range(len(prompts)))
        self.outs = [[] for _ in prompts]
        pg = getattr(m, "pager", None)
        if pg is not None:
            # paged compressed caches: each sequence holds blocks for the whole context
            for s in range(pg.n_slots - 1):      # the speculative engine owns every slot of the model
                pg.release(s)
            for s in self.slots:
                if not pg.reserve(s, m.max_seq_len):
                    raise ValueError("paged cache pool too small for the speculative sequences")
        for j, p in enumerate(prompts):
            for c0 in range(0, len(p), m.max_tokens):
                piece = p[c0:c0 + m.max_tokens]
                last = c0 + len(piece) == len(p)
                meta = StepMeta(cfg, [SeqChunk(self.slots[j], c0, piece, last)])
                ids = self._run(meta, taps=dr.taps)
                dr.ingest(None, meta.T)
                if last:
                    self.outs[j].append(int(ids[0]))
        self.pos = [len(p) for p in prompts]       # position of each root

    def draft(self, act: list[int]) -> np.ndarray:
        """Drafts for sequences ``act``; returns toks [blk+1, len(act)] (row 0 = roots)."""
        m, cfg, dr = self.m, self.cfg, self.drafter
        na = len(act)
        dmeta = StepMeta(cfg, [SeqChunk(self.slots[j], self.pos[j], [self.outs[j][-1]] +
                                        [cfg.dspark_noise_token_id] * (self.blk - 1), True, True) for j in act])
        m.upload(dmeta, self.pinned)
        m._last_meta = dmeta
        dr.toks[0, :na].copy_(torch.tensor([self.outs[j][-1] for j in act], dtype=torch.int32))
        return dr.draft(na).cpu().numpy()

    # ------------------------------------------------------- per-row serving
    def open_rows(self) -> None:
        """Per-row state for serving (rows admitted and released one by one)."""
        self.slots = list(range(self.max_seqs))
        self.outs = [[] for _ in range(self.max_seqs)]
        self.pos = [0] * self.max_seqs

    def add_sequence(self, j: int, prompt: list[int]) -> int:
        """Prefills ``prompt`` (chunked) into row ``j`` (model slot ``j``) and fills the
        MTP rings; returns the first generated token."""
        m, cfg, dr = self.m, self.cfg, self.drafter
        pg = getattr(m, "pager", None)
        if pg is not None and not pg.reserve(self.slots[j], m.max_seq_len):
            raise ValueError("paged cache pool has no room for another speculative sequence")
        first = None
        for c0 in range(0, len(prompt), m.max_tokens):
            piece = prompt[c0:c0 + m.max_tokens]
            last = c0 + len(piece) == len(prompt)
            meta = StepMeta(cfg, [SeqChunk(self.slots[j], c0, piece, last)])
            ids = self._run(meta, taps=dr.taps)
            dr.ingest(None, meta.T)
            if last:
                first = int(ids[0])
        self.outs[j] = [first]
        self.pos[j] = len(prompt)
        return first

    def release_row(self, j: int) -> None:
        pg = getattr(self.m, "pager", None)
        if pg is not None:
            pg.release(self.slots[j])
        self.outs[j] = []

    def round(self, act: list[int], limits: list[int]) -> list[list[int]]:
        """One draft + verify round for rows ``act`` (``limits``: output length cap
        per row); returns the tokens each row emitted."""
        before = [len(self.outs[j]) for j in act]
        toks = self.draft(act)
        blocks = [[self.outs[j][-1]] + [int(toks[i + 1, a]) for i in range(self.blk - 1)]
                  for a, j in enumerate(act)]
        self.verify(act, blocks, limits)
        return [self.outs[j][b:] for j, b in zip(act, before)]

    def verify(self, act: list[int], blocks: list[list[int]], max_new_tokens=None) -> list[int]:
        """Verifies blocks [root, d1..d_{B-1}] per sequence; commits, ingests, emits.

        ``max_new_tokens``: output length cap, one for all rows or a list per row
        of ``act``.  Returns the accepted draft count per sequence."""
        m, cfg, dr = self.m, self.cfg, self.drafter
        na = len(act)
        vmeta = StepMeta(cfg, [SeqChunk(self.slots[j], self.pos[j], blocks[a], True, True) for a, j in enumerate(act)])
        preds = self._run(vmeta, taps=dr.taps, defer_rings=True).cpu().numpy().reshape(na, self.blk)
        n_acc = []
        for a in range(na):
            if self.force_accept is not None:
                f = float(self.force_accept)
                r = self._forced_rounds
                self._forced_rounds += 1
                k = min(int(math.floor((r + 1) * f + 1e-9) - math.floor(r * f + 1e-9)), self.blk - 1)
            else:
                k = 0
                while k < self.blk - 1 and preds[a, k] == blocks[a][k + 1]:
                    k += 1
            n_acc.append(k)
        # rings keep positions <= pos + n_acc only
        last = np.repeat([self.pos[j] + n_acc[a] for a, j in enumerate(act)], self.blk).astype(np.int32)
        m.commit_rings(vmeta.T, torch.from_numpy(last).to(m.dev))
        # the accepted rows' main hidden enters every stage ring
        rows = np.concatenate([a * self.blk + np.arange(n_acc[a] + 1) for a in range(na)]).astype(np.int64)
        imeta = self._ingest_meta([self.slots[j] for j in act], [k + 1 for k in n_acc], [self.pos[j] for j in act])
        m.upload(imeta, self.pinned)
        dr.ingest(torch.from_numpy(rows).to(m.dev), imeta.T)
        for a, j in enumerate(act):
            k = n_acc[a]
            emitted = blocks[a][1:k + 1] + [int(preds[a, k])]
            cap = max_new_tokens[a] if isinstance(max_new_tokens, (list, tuple)) else max_new_tokens
            room = len(emitted) if cap is None else cap - len(self.outs[j])
            self.outs[j].extend(emitted[:room])
            self.pos[j] += k + 1
            self.stats.rounds += 1
            self.stats.drafted += self.blk - 1
            self.stats.accepted += k
            self.stats.emitted += min(len(emitted), room)
            self.stats.histogram[k] += 1
        return n_acc

    def generate(self, prompts: list[list[int]], max_new_tokens: int) -> list[list[int]]:
        self.prefill(prompts)
        while True:
            act = [j for j in range(len(prompts)) if len(self.outs[j]) < max_new_tokens]
            if not act:
                break
            toks = self.draft(act)
            blocks = [[self.outs[j][-1]] + [int(toks[i + 1, a]) for i in range(self.blk - 1)]
                      for a, j in enumerate(act)]
            self.verify(act, blocks, max_new_tokens)
        return self.outs
