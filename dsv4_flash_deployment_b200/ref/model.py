"""CPU oracle of the DeepSeek-V4 family forward pass (token-sequential).

A direct statement of the decode math of the reference oracle
(``models/DeepSeekV4.1-Flash-v6e16/tpu-v7x/deepseek_v41/reference.py``):
block structure ``_block_step`` (``:840-891``), attention ``_attention_step``
(``:704-838``), compressor ``_compressor_step`` (``:547-603``), indexer
``_indexer_step`` (``:605-702``), MoE ``moe_forward`` (``:355-423``), Engram
``engram_forward`` (``:272-319``), DSpark ``forward_spec`` (``:1116-1248``) and
``verify_block`` (``:1250-1329``).

Prefill is run as consecutive single-token steps; the reference states that a
prefill or verify block has exactly the semantics of sequential decode steps,
so one code path is the whole oracle.  All B rows of a batch sit at the same
position.  V4-Flash-shaped configs add: q per-head RMSNorm, compressor gate
position embedding, 2-group overlapped compressor windows and dense (no
indexer) attention over the compressed cache for layers that own a compressor
but no indexer.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field

import numpy as np
import torch

from . import numerics as N
from .engram import EngramHasher


@dataclass
class RefState:
    batch: int
    pos: int = 0
    window: dict[int, torch.Tensor] = field(default_factory=dict)        # [B, W, d] bf16 ring
    comp_kv: dict[int, list[torch.Tensor]] = field(default_factory=dict)  # list of [B, d] bf16
    index_k: dict[int, list[torch.Tensor]] = field(default_factory=dict)  # list of [B, dk] bf16
    proj_hist: dict[int, list[tuple[torch.Tensor, torch.Tensor]]] = field(default_factory=dict)
    shared_index_k_source: int | None = None
    engram_hist: list[np.ndarray] = field(default_factory=list)          # per row: compressed ids

    def clone(self) -> "RefState":
        return copy.deepcopy(self)


class RefModel:
    def __init__(self, cfg, weights: dict[str, torch.Tensor], max_seq_len: int = 512,
                 sinkhorn_iters: int | None = None, index_k_mode: str | None = None):
        self.cfg = cfg
        self.w = weights
        self.max_seq_len = max_seq_len
        self.sinkhorn_iters = cfg.hc_sinkhorn_iters if sinkhorn_iters is None else sinkhorn_iters
        self.index_k_mode = index_k_mode or cfg.index_k_mode
        self.rope = N.layer_rope_tables(cfg, max_seq_len + 16)
        self.hasher = EngramHasher(cfg) if cfg.engram_layer_ids else None

    # ------------------------------------------------------------------ state
    def new_state(self, batch: int) -> RefState:
        cfg = self.cfg
        st = RefState(batch=batch)
        for lid in range(cfg.n_total_layers):
            st.window[lid] = torch.zeros(batch, cfg.sliding_window, cfg.head_dim, dtype=torch.bfloat16)
        for lid in cfg.kv_source_layer_ids:
            st.comp_kv[lid] = []
            st.index_k[lid] = []
            st.proj_hist[lid] = []
        st.engram_hist = [np.zeros(0, np.int64) for _ in range(batch)]
        return st

    def _rope(self, lid: int, pos: int):
        key = "yarn" if (lid < self.cfg.n_layers and self.cfg.ratio(lid) > 0) else "swa"
        c, s = self.rope[key]
        return c[pos], s[pos]

    def _mixes(self, h, prefix, which):
        cfg = self.cfg
        return N.hc_mixes(h, self.w[f"{prefix}.hc_{which}_fn"], self.w[f"{prefix}.hc_{which}_scale"],
                          self.w[f"{prefix}.hc_{which}_base"], cfg.hc_mult, self.sinkhorn_iters,
                          cfg.hc_eps, cfg.rms_norm_eps)

    def _lin(self, x, name):
        return N.fp8_linear(x, self.w[f"{name}.weight"], self.w[f"{name}.scale"])

    # ------------------------------------------------------------- compressor
    def _compressor(self, lid: int, u: torch.Tensor, pos: int, st: RefState):
        """Pooled latent [B, d] when position ``pos`` closes a group, else None."""
        cfg = self.cfg
        r = cfg.ratio(lid)
        co = cfg.overlap(lid)
        d = cfg.head_dim
        p = f"layers.{lid}.attn.compressor"
        kv = u.float() @ self.w[f"{p}.wkv.weight"].float().t()                 # [B, co*d]
        if r > 1:
            sc = u.float() @ self.w[f"{p}.wgate.weight"].float().t()
            if cfg.compressor_ape:
                sc = sc + self.w[f"{p}.ape"].float()[pos % r]
        else:
            sc = torch.zeros_like(kv)
        st.proj_hist[lid].append((kv, sc))
        if (pos + 1) % r:
            return None
        g = pos // r
        kvs, scs = [], []
        hist = st.proj_hist[lid]
        if co == 2:
            for t in range((g - 1) * r, g * r):
                if t >= 0:
                    kvs.append(hist[t][0][:, :d]); scs.append(hist[t][1][:, :d])
        for t in range(g * r, (g + 1) * r):
            kvs.append(hist[t][0][:, (co - 1) * d:]); scs.append(hist[t][1][:, (co - 1) * d:])
        kv_s = torch.stack(kvs, 1)
        sc_s = torch.stack(scs, 1)
        pooled = (kv_s * torch.softmax(sc_s, 1)).sum(1)
        return N.rms_norm(pooled.to(torch.bfloat16), self.w[f"{p}.norm.weight"], cfg.rms_norm_eps)

    # ---------------------------------------------------------------- indexer
    def _indexer(self, lid, u, qr, latent, pos, st: RefState, rt: dict) -> torch.Tensor:
        cfg = self.cfg
        r = cfg.ratio(lid)
        p = f"layers.{lid}.attn.indexer"
        clen = (pos + 1) // r
        if lid in cfg.kv_source_layer_ids and latent is not None:
            c, s = self._rope(lid, pos + 1 - r)
            k = N.rms_norm(N.bf16_linear(latent, self.w[f"{p}.wk.weight"]), self.w[f"{p}.k_norm.weight"],
                           cfg.rms_norm_eps)
            k = N.apply_rope(k, c, s)
            k = N.fp4_act_quant_roundtrip(k, 32, "e8m0")
            st.index_k[lid].append(k)
            st.shared_index_k_source = lid
        if self.index_k_mode == "intended":
            src = cfg.kv_source_for(lid)
        else:
            src = st.shared_index_k_source if st.shared_index_k_source is not None else cfg.kv_source_for(lid)
        kcache = torch.stack(st.index_k[src][:clen], 1)                         # [B, T, dk]
        q = self._lin(qr, f"{p}.wq_b").reshape(st.batch, cfg.index_n_heads, cfg.index_head_dim)
        c, s = self._rope(lid, pos)
        q = N.apply_rope(q, c, s)
        q = N.fp4_act_quant_roundtrip(q, 32, "e8m0")
        sw = (cfg.index_head_dim ** -0.5) * (cfg.index_n_heads ** -0.5)
        wts = (N.bf16_linear(u, self.w[f"{p}.weights_proj.weight"]).float() * sw).to(torch.bfloat16)
        raw = torch.einsum("bhd,btd->bht", q.float(), kcache.float()).to(torch.bfloat16)
        gated = (raw.clamp_min(0).float() * wts[..., None].float()).to(torch.bfloat16)
        score = gated.float().sum(1).to(torch.bfloat16)                          # [B, T]
        if lid == cfg.candidate_source_layer_id:
            rt["candidates"] = N.select_candidate_blocks(score, torch.tensor(clen),
                                                         cfg.candidate_topk_blocks, cfg.candidate_block_size)
        elif 0 <= cfg.candidate_source_layer_id < lid:
            cand = rt["candidates"]
            width = score.shape[-1]
            if cand.shape[-1] < width:  # the mask was built at an earlier, shorter length
                cand = torch.nn.functional.pad(cand, (0, width - cand.shape[-1]), value=False)
            score = torch.where(cand[..., :width], score, torch.tensor(float("-inf"), dtype=score.dtype))
        kk = min(cfg.index_topk, clen)
        _, top = torch.topk(score.float(), kk, -1)
        top, _ = torch.sort(top, -1)
        return torch.where(top < clen, top + cfg.sliding_window, torch.full_like(top, -1))

    # -------------------------------------------------------------- attention
    def _attention(self, lid: int, u: torch.Tensor, pos: int, st: RefState, rt: dict) -> torch.Tensor:
        cfg = self.cfg
        b = st.batch
        p = f"layers.{lid}.attn"
        c, s = self._rope(lid, pos)
        qr = N.rms_norm(self._lin(u, f"{p}.wq_a"), self.w[f"{p}.q_norm.weight"], cfg.rms_norm_eps)
        q = self._lin(qr, f"{p}.wq_b").reshape(b, cfg.n_heads, cfg.head_dim)
        if cfg.q_head_norm:
            qf = q.float()
            q = (qf * torch.rsqrt(qf.square().mean(-1, keepdim=True) + cfg.rms_norm_eps)).to(q.dtype)
        q = N.apply_rope(q, c, s)
        kv = N.rms_norm(self._lin(u, f"{p}.wkv"), self.w[f"{p}.kv_norm.weight"], cfg.rms_norm_eps)
        kv = N.apply_rope(kv, c, s)
        kv = N.act_quant_roundtrip(kv)
        W = cfg.sliding_window
        st.window[lid][:, pos % W] = kv
        win_idx = torch.arange(W)
        win_idx = torch.where(win_idx <= pos, win_idx, torch.full_like(win_idx, -1))
        idx = win_idx[None].expand(b, W)
        kv_all = st.window[lid]
        r = cfg.ratio(lid)
        if r > 0:
            clen = (pos + 1) // r
            latent = None
            if lid in cfg.kv_source_layer_ids:
                latent = self._compressor(lid, u, pos, st)
                rt["kv_source"] = lid
            if lid in cfg.index_source_layer_ids:
                cidx = (self._indexer(lid, u, qr, latent, pos, st, rt) if clen > 0
                        else torch.zeros(b, 0, dtype=torch.long))
                rt["topk"] = cidx
            elif lid in cfg.kv_source_layer_ids:
                cidx = (torch.arange(clen) + W)[None].expand(b, clen)
            else:
                cidx = rt["topk"]
            if latent is not None:
                gc, gs = self._rope(lid, pos + 1 - r)
                lat = N.apply_rope(latent, gc, gs)
                st.comp_kv[lid].append(N.fp4_act_quant_roundtrip(lat, 16, "e4m3"))
            src = rt["kv_source"]
            if clen > 0:
                kv_all = torch.cat([kv_all, torch.stack(st.comp_kv[src][:clen], 1)], 1)
            idx = torch.cat([idx, cidx], -1)
        o = N.sparse_attn(q[:, None], kv_all, self.w[f"{p}.attn_sink"], idx[:, None], cfg.head_dim ** -0.5)[:, 0]
        o = N.apply_rope(o, c, s, inverse=True)
        return self._o_proj(o, p)

    def _o_proj(self, o: torch.Tensor, p: str) -> torch.Tensor:
        cfg = self.cfg
        lead = o.shape[:-2]
        og = o.reshape(*lead, cfg.o_groups, -1)
        wo_a = N.dequant_fp8_block(self.w[f"{p}.wo_a.weight"], self.w[f"{p}.wo_a.scale"]).to(torch.bfloat16)
        wo_a = wo_a.reshape(cfg.o_groups, cfg.o_lora_rank, -1)
        proj = torch.einsum("...gd,grd->...gr", og.float(), wo_a.float()).to(torch.bfloat16)
        return self._lin(proj.reshape(*lead, cfg.o_inter), f"{p}.wo_b")

    # --------------------------------------------------------------------- MoE
    def _moe(self, lid: int, x: torch.Tensor, prefix: str) -> torch.Tensor:
        cfg = self.cfg
        ids, wts = N.route(x, self.w[f"{prefix}.ffn.gate.weight"], self.w[f"{prefix}.ffn.gate.bias"],
                           cfg.topk_for(lid), cfg.route_scale, cfg.score_func)
        y = torch.zeros(x.shape[0], cfg.dim)
        for e in torch.unique(ids).tolist():
            tok, slot = torch.nonzero(ids == e, as_tuple=True)
            ep = f"{prefix}.ffn.experts.{e}"
            y.index_add_(0, tok, N.expert_ffn(
                x[tok], self.w[f"{ep}.w1.weight"], self.w[f"{ep}.w1.scale"], self.w[f"{ep}.w3.weight"],
                self.w[f"{ep}.w3.scale"], self.w[f"{ep}.w2.weight"], self.w[f"{ep}.w2.scale"],
                cfg.swiglu_limit, wts[tok, slot][:, None]))
        sp = f"{prefix}.ffn.shared_experts"
        shared = N.expert_ffn(x, self.w[f"{sp}.w1.weight"], self.w[f"{sp}.w1.scale"], self.w[f"{sp}.w3.weight"],
                              self.w[f"{sp}.w3.scale"], self.w[f"{sp}.w2.weight"], self.w[f"{sp}.w2.scale"],
                              cfg.swiglu_limit)
        return (y + shared).to(torch.bfloat16)

    # ----------------------------------------------------------------- Engram
    def engram_rows(self, lid: int, hash_ids: torch.Tensor) -> torch.Tensor:
        """Gathered, dequantized, masked rows flattened to [B, n_cols*head_dim] bf16."""
        cfg = self.cfg
        i = cfg.engram_layer_ids.index(lid)
        n_emb = cfg.engram_num_embeddings[i]
        p = f"layers.{lid}.engram"
        mask = (hash_ids < 0) | (hash_ids >= n_emb)
        safe = torch.where(mask, torch.zeros_like(hash_ids), hash_ids)
        vals = N.dequant_fp8_block(self.w[f"{p}.embed.weight"][safe].reshape(-1, cfg.engram_head_dim),
                                   self.w[f"{p}.embed.scale"][safe].reshape(-1, cfg.engram_head_dim // 32))
        vals = vals.reshape(*safe.shape, cfg.engram_head_dim).to(torch.bfloat16)
        vals = torch.where(mask[..., None], torch.zeros((), dtype=torch.bfloat16), vals)
        return vals.reshape(*safe.shape[:-1], -1)

    def _engram(self, lid: int, h: torch.Tensor, hash_ids: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        p = f"layers.{lid}.engram"
        flat = self.engram_rows(lid, hash_ids)
        kv = self._lin(flat, f"{p}.wkv")
        hd = cfg.hc_mult * cfg.dim
        key = kv[..., :hd].float().reshape(*h.shape[:-2], cfg.hc_mult, cfg.dim)
        value = kv[..., hd:]
        wgt = self.w[f"{p}.q_weight"].float() * self.w[f"{p}.k_weight"].float()
        hf = h.float()
        eps = cfg.rms_norm_eps
        rstd = torch.rsqrt(hf.square().mean(-1) + eps) * torch.rsqrt(key.square().mean(-1) + eps)
        dot = (hf * wgt * key).sum(-1) * rstd * cfg.dim ** -0.5
        g = torch.sigmoid(torch.copysign(torch.sqrt(dot.abs().clamp_min(1e-6)), dot))
        return (hf + g[..., None] * value.float()[..., None, :]).to(h.dtype)

    def engram_hashes(self, ids: torch.Tensor, pos: int, st: RefState) -> torch.Tensor:
        """Row ids [B, n_engram_layers, n_cols] for tokens ``ids`` [B] at ``pos``."""
        out = []
        for b in range(st.batch):
            hist = st.engram_hist[b]
            if len(hist) <= pos:
                hist = np.concatenate([hist, np.zeros(pos + 1 - len(hist), np.int64)])
            hist[pos] = self.hasher.compress([int(ids[b])])[0]
            st.engram_hist[b] = hist
            out.append(self.hasher.hash(hist[: pos + 1], np.array([pos]))[0])
        return torch.from_numpy(np.stack(out))

    # ---------------------------------------------------------------- forward
    def _block(self, lid: int, h, pre_mix, pos, st, rt, prefix=None):
        cfg = self.cfg
        p = prefix or f"layers.{lid}"
        a_pre, a_post, a_comb = self._mixes(h, p, "attn")
        u = N.rms_norm(N.hc_pre(h, pre_mix), self.w[f"{p}.attn_norm.weight"], cfg.rms_norm_eps)
        att = self._attention(lid, u, pos, st, rt) if prefix is None else rt["dspark_attn"](lid, u)
        h = N.hc_post(att, h, a_post, a_comb)
        f_pre, f_post, f_comb = self._mixes(h, p, "ffn")
        v = N.rms_norm(N.hc_pre(h, a_pre), self.w[f"{p}.ffn_norm.weight"], cfg.rms_norm_eps)
        h = N.hc_post(self._moe(lid, v, p), h, f_post, f_comb)
        return h, f_pre

    def step(self, ids: torch.Tensor, st: RefState, trace: dict | None = None):
        """One decode step for tokens ``ids`` [B] at ``st.pos``.

        Returns (logits [B, V] fp32, main_hidden [B, n_taps*D] bf16 or None).
        """
        cfg = self.cfg
        pos = st.pos
        b = ids.shape[0]
        hashes = self.engram_hashes(ids, pos, st) if self.hasher is not None else None
        h = self.w["embed.weight"][ids].to(torch.bfloat16)[:, None, :].repeat(1, cfg.hc_mult, 1)
        pre_mix = torch.zeros(b, cfg.hc_mult)
        pre_mix[:, 0] = 1.0
        rt: dict = {}
        taps = []
        for lid in range(cfg.n_layers):
            if cfg.has_engram(lid):
                h = self._engram(lid, h, hashes[:, cfg.engram_layer_ids.index(lid)])
            if lid in cfg.dspark_target_layer_ids:
                taps.append(h.float().mean(-2).to(torch.bfloat16))
            if trace is not None:
                trace.setdefault(lid, []).append(h.clone())
            h, pre_mix = self._block(lid, h, pre_mix, pos, st, rt)
        y = N.rms_norm(N.hc_pre(h, pre_mix), self.w["norm.weight"], cfg.rms_norm_eps)
        logits = y.float() @ self.w["head.weight"].float().t()
        st.pos += 1
        return logits, (torch.cat(taps, -1) if taps else None)

    def generate(self, prompt: torch.Tensor, n_new: int, st: RefState | None = None):
        """Greedy: prompt [B, S] -> generated [B, n_new]."""
        st = st or self.new_state(prompt.shape[0])
        logits = None
        for t in range(prompt.shape[1]):
            logits, _ = self.step(prompt[:, t], st)
        out = []
        for _ in range(n_new):
            nxt = logits.argmax(-1)
            out.append(nxt)
            logits, _ = self.step(nxt, st)
        return torch.stack(out, 1), st

    # ----------------------------------------------------------------- DSpark
    def dspark_state_init(self, st: RefState) -> None:
        st.dspark_pos = 0  # number of main-hidden rows written into the DSpark rings

    def _dspark_main_x(self, main_hidden: torch.Tensor) -> torch.Tensor:
        return N.rms_norm(self._lin(main_hidden, "mtp.0.main_proj"), self.w["mtp.0.main_norm.weight"],
                          self.cfg.rms_norm_eps)

    def dspark_ingest(self, main_hidden: torch.Tensor, start_pos: int, st: RefState) -> None:
        """Writes main-hidden rows for target positions start_pos.. into every stage's ring."""
        cfg = self.cfg
        mx = self._dspark_main_x(main_hidden)                                   # [B, s, D]
        for k in range(cfg.n_mtp_layers):
            lid = cfg.n_layers + k
            p = f"mtp.{k}.attn"
            kv = N.rms_norm(self._lin(mx, f"{p}.wkv"), self.w[f"{p}.kv_norm.weight"], cfg.rms_norm_eps)
            for i in range(mx.shape[1]):
                c, s = self._rope(lid, start_pos + i)
                row = N.act_quant_roundtrip(N.apply_rope(kv[:, i], c, s))
                st.window[lid][:, (start_pos + i) % cfg.sliding_window] = row

    def draft(self, root: torch.Tensor, main_hidden: torch.Tensor, start_pos: int, st: RefState):
        """DSpark draft (``forward_spec`` at start_pos > 0).

        main_hidden [B, s, 3D] holds the taps of target positions
        start_pos..start_pos+s-1; ``root`` [B] is the token at start_pos+s.
        Returns (tokens [B, block+1] = root + block predictions, logits, confidence).
        """
        cfg = self.cfg
        b = root.shape[0]
        s_len = main_hidden.shape[1]
        self.dspark_ingest(main_hidden, start_pos, st)
        blk = cfg.dspark_block_size
        W = cfg.sliding_window
        d0 = start_pos + s_len
        ring_valid = min(W, d0)
        ids = torch.full((b, blk), cfg.dspark_noise_token_id, dtype=torch.long)
        ids[:, 0] = root
        h = self.w["embed.weight"][ids].to(torch.bfloat16)[:, :, None, :].repeat(1, 1, cfg.hc_mult, 1)
        pre_mix = torch.zeros(b, blk, cfg.hc_mult)
        pre_mix[..., 0] = 1.0

        def attn(lid: int, u: torch.Tensor) -> torch.Tensor:
            p = f"mtp.{lid - cfg.n_layers}.attn"
            cos = torch.stack([self._rope(lid, d0 + i)[0] for i in range(blk)])
            sin = torch.stack([self._rope(lid, d0 + i)[1] for i in range(blk)])
            qr = N.rms_norm(self._lin(u, f"{p}.wq_a"), self.w[f"{p}.q_norm.weight"], cfg.rms_norm_eps)
            q = self._lin(qr, f"{p}.wq_b").reshape(b, blk, cfg.n_heads, cfg.head_dim)
            q = N.apply_rope(q, cos[:, None], sin[:, None])
            kv = N.rms_norm(self._lin(u, f"{p}.wkv"), self.w[f"{p}.kv_norm.weight"], cfg.rms_norm_eps)
            kv = N.act_quant_roundtrip(N.apply_rope(kv, cos, sin))
            kv_all = torch.cat([st.window[lid], kv], 1)
            idx = torch.cat([torch.arange(ring_valid), W + torch.arange(blk)])[None, None].expand(b, blk, -1)
            o = N.sparse_attn(q, kv_all, self.w[f"{p}.attn_sink"], idx, cfg.head_dim ** -0.5)
            o = N.apply_rope(o, cos[:, None], sin[:, None], inverse=True)
            return self._o_proj(o, p)

        rt = {"dspark_attn": attn}
        for k in range(cfg.n_mtp_layers):
            lid = cfg.n_layers + k
            hb = h.reshape(b * blk, cfg.hc_mult, cfg.dim)
            pm = pre_mix.reshape(b * blk, cfg.hc_mult)
            # mixes/norm/MoE are per token: flatten the block, attention sees [B, blk].
            prefix = f"mtp.{k}"
            a_pre, a_post, a_comb = self._mixes(hb, prefix, "attn")
            u = N.rms_norm(N.hc_pre(hb, pm), self.w[f"{prefix}.attn_norm.weight"], cfg.rms_norm_eps)
            att = attn(lid, u.reshape(b, blk, cfg.dim)).reshape(b * blk, cfg.dim)
            hb = N.hc_post(att, hb, a_post, a_comb)
            f_pre, f_post, f_comb = self._mixes(hb, prefix, "ffn")
            v = N.rms_norm(N.hc_pre(hb, a_pre), self.w[f"{prefix}.ffn_norm.weight"], cfg.rms_norm_eps)
            hb = N.hc_post(self._moe(lid, v, prefix), hb, f_post, f_comb)
            h = hb.reshape(b, blk, cfg.hc_mult, cfg.dim)
            pre_mix = f_pre.reshape(b, blk, cfg.hc_mult)
        last = f"mtp.{cfg.n_mtp_layers - 1}"
        xc = N.hc_pre(h, pre_mix)
        normed = N.rms_norm(xc, self.w[f"{last}.norm.weight"], cfg.rms_norm_eps)
        logits = normed.float() @ self.w["head.weight"].float().t()
        memb = self.w[f"{last}.markov_head.embed.weight"].to(torch.bfloat16)
        mhead = self.w[f"{last}.markov_head.head.weight"].float()
        toks = [root]
        out_logits, embs = [], []
        for i in range(blk):
            e = memb[toks[i]]
            li = logits[:, i] + e.float() @ mhead.t()
            toks.append(li.argmax(-1))
            out_logits.append(li)
            embs.append(e)
        conf_in = torch.cat([xc, torch.stack(embs, 1)], -1).float()
        conf = (conf_in @ self.w[f"{last}.confidence_head.proj.weight"].float().t())[..., 0]
        return torch.stack(toks, 1), torch.stack(out_logits, 1), conf

    def verify(self, block_ids: torch.Tensor, st: RefState, force_accept: int | None = None):
        """Verify [B=1, q] = [root, drafts...] at st.pos (``reference.py:1250-1329``).

        Commits the state after n_accepted+1 tokens and returns a dict with the
        emitted tokens (accepted drafts + bonus) and their main hiddens.
        """
        q = block_ids.shape[1]
        work = st.clone()
        states, preds, hiddens, logits_all = [], [], [], []
        for i in range(q):
            lg, mh = self.step(block_ids[:, i], work)
            states.append(work.clone())
            preds.append(int(lg.argmax(-1)[0]))
            hiddens.append(mh)
            logits_all.append(lg)
        if force_accept is not None:
            n_acc = int(force_accept)
        else:
            n_acc = 0
            for i in range(q - 1):
                if preds[i] == int(block_ids[0, i + 1]):
                    n_acc += 1
                else:
                    break
        committed = states[n_acc]
        st.__dict__.update(committed.__dict__)
        emitted = [int(block_ids[0, i]) for i in range(1, n_acc + 1)] + [preds[n_acc]]
        mh = torch.stack(hiddens[: n_acc + 1], 1) if hiddens[0] is not None else None
        return {"num_accepted": n_acc, "emitted": emitted, "bonus": preds[n_acc],
                "main_hidden": mh, "logits": torch.stack(logits_all, 1)}
